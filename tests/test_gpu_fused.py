"""ecq_gemv_fused: the batch-1 GEMV with the decode step's element-wise
follower fused into its epilogue (RoPE + KV-cache store after q|k|v, SwiGLU
after gate|up), against the same GEMV followed by the separate glue kernel
(ecq_rope_kv_f16 / ecq_silu_mul_f16) and against the float64 oracle."""
import numpy as np
import pytest

from oracle import oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import ecq_b200 as ecq  # noqa: E402
from ecq_b200 import _lib  # noqa: E402
from ecq_b200 import synthetic as syn  # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _ulp_close(a, b, ulps=1):
    """fp16 tensors equal to within `ulps` units in the last place."""
    a16 = a.contiguous().view(torch.int16).int()
    b16 = b.contiguous().view(torch.int16).int()
    return int((a16 - b16).abs().max()) <= ulps


@pytest.mark.parametrize("heads,D,K,tc", [(4, 128, 512, 512), (8, 128, 1024, 256), (2, 64, 256, 128)])
def test_gemv_rope_kv_matches_gemv_then_rope(heads, D, K, tc):
    L = heads * D
    M = 3 * L
    sym = syn.laplace_symbols(M, K, b=0.5, seed=heads + D)
    sc = torch.from_numpy(syn.group_scales(M, K, 128 if tc >= 128 else 64, seed=3)).cuda()
    m = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(sym, tile_cols=tc, group_size=128), group_size=128)
    x = torch.from_numpy(syn.activations(1, K, seed=4)).cuda()
    ang = 2049.0 / (10000.0 ** (torch.arange(0, D, 2, device="cuda", dtype=torch.float32) / D))
    cos, sin = torch.cos(ang).half(), torch.sin(ang).half()
    T = 70
    kv_ref = torch.randn(2, heads, T, D, device="cuda").half()
    kv = kv_ref.clone()
    # reference: plain GEMV, then the rope_kv glue kernel
    y_ref = m.gemv(x, sc).clone()
    st = torch.cuda.current_stream().cuda_stream
    assert _lib.lib().ecq_rope_kv_f16(y_ref.data_ptr(), y_ref[:, L:].data_ptr(), y_ref[:, 2 * L:].data_ptr(),
                                      kv_ref[0, :, T - 1].data_ptr(), kv_ref[1, :, T - 1].data_ptr(),
                                      cos.data_ptr(), sin.data_ptr(), heads, D, T * D, st) == 0
    y = m.gemv_rope_kv(x, sc, cos, sin, kv[0, :, T - 1], kv[1, :, T - 1], D, T * D)
    torch.cuda.synchronize()
    m.check()
    assert _ulp_close(y[:, :L], y_ref[:, :L])                  # q rotated
    assert torch.equal(y[:, 2 * L:], y_ref[:, 2 * L:])         # v as the GEMV gives it
    assert _ulp_close(kv, kv_ref)                              # the cache slot (and nothing else) written
    assert torch.equal(kv[:, :, :T - 1], kv_ref[:, :, :T - 1])


@pytest.mark.parametrize("F,K,tc", [(512, 1024, 512), (1376, 4096, 256), (72, 256, 128)])
def test_gemv_silu_mul_matches_gemv_then_silu(F, K, tc):
    g_sym = syn.laplace_symbols(F, K, b=1.0, seed=F)
    u_sym = syn.laplace_symbols(F, K, b=1.0, seed=F + 1)
    g_sc = syn.group_scales(F, K, 128, seed=5)
    u_sc = syn.group_scales(F, K, 128, seed=6)
    inter = np.stack([g_sym, u_sym], axis=1).reshape(2 * F, K)
    inter_sc = np.stack([g_sc, u_sc], axis=1).reshape(2 * F, -1)
    m = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(inter, tile_cols=tc, group_size=128), group_size=128)
    x = torch.from_numpy(syn.activations(1, K, seed=7)).cuda()
    s = torch.from_numpy(inter_sc).cuda()
    y = m.gemv(x, s)
    gu = torch.cat([y[:, 0::2], y[:, 1::2]], dim=1).contiguous()  # gate | up, as ecq_silu_mul_f16 reads it
    ref = torch.empty(1, F, dtype=torch.float16, device="cuda")
    assert _lib.lib().ecq_silu_mul_f16(gu.data_ptr(), ref.data_ptr(), F, 1, torch.cuda.current_stream().cuda_stream) == 0
    out = m.gemv_silu_mul(x, s)
    torch.cuda.synchronize()
    m.check()
    assert out.shape == (1, F) and _ulp_close(out, ref)
    g64 = oracle.dequant_gemv(g_sym, g_sc.astype(np.float32), 128, x.float().cpu().numpy())
    u64 = oracle.dequant_gemv(u_sym, u_sc.astype(np.float32), 128, x.float().cpu().numpy())
    m64 = g64.astype(np.float64) / (1.0 + np.exp(-g64.astype(np.float64))) * u64
    err = float(np.max(np.abs(out.float().cpu().numpy()[0] - m64)) / np.max(np.abs(m64)))
    assert err <= 5e-3


def test_gemv_fused_argument_errors():
    m = ecq.DeviceMatrix.from_encoded(ecq.encode_matrix(syn.laplace_symbols(24, 512, b=0.5, seed=1), group_size=128),
                                      group_size=128)
    x = torch.zeros(1, 512, dtype=torch.float16, device="cuda")
    s = torch.zeros(24, 4, dtype=torch.float16, device="cuda")
    y = torch.zeros(1, 24, dtype=torch.float16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    P = _lib.ptr
    bad = _lib.GemvEpilogue(kind=7)
    assert _lib.lib().ecq_gemv_fused(m.view(), P(x), P(s), P(y), bad, P(m.workspace), m.workspace.numel(),
                                     P(m.status), st) == -1
    rope = _lib.GemvEpilogue(kind=_lib.EPI_ROPE_KV, part_rows=8, head_dim=3, cache_head_stride=8,
                             cos_f16=16, sin_f16=16, k_cache_f16=16, v_cache_f16=16)  # odd head_dim
    assert _lib.lib().ecq_gemv_fused(m.view(), P(x), P(s), P(y), rope, P(m.workspace), m.workspace.numel(),
                                     P(m.status), st) == -1


@pytest.mark.parametrize("rows,n,with_d", [(1, 4096, True), (1, 4096, False), (1, 11008, True), (3, 4096, True),
                                           (1, 512, True), (1, 1031, True)])
def test_add_rmsnorm_against_reference(rows, n, with_d):
    # one row of n >= 1024 runs on a cluster of 8 CTAs, everything else one CTA per row
    g = torch.Generator(device="cuda").manual_seed(rows * n)
    h = torch.randn(rows, n, device="cuda", generator=g).half()
    d = torch.randn(rows, n, device="cuda", generator=g).half() if with_d else None
    w = (1 + 0.1 * torch.randn(n, device="cuda", generator=g)).half()
    h0 = h.clone()
    y = torch.empty_like(h)
    assert _lib.lib().ecq_add_rmsnorm_f16(h.data_ptr(), d.data_ptr() if with_d else None, w.data_ptr(), h.data_ptr(),
                                          y.data_ptr(), rows, n, 1e-5, torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    hr = (h0.float() + d.float()).half().float() if with_d else h0.float()
    yr = (hr * torch.rsqrt(hr.pow(2).mean(-1, keepdim=True) + 1e-5)).half().float() * w.float()
    if with_d:
        assert torch.equal(h.float(), hr)  # the residual, in place
    assert float((y.float() - yr).abs().max() / yr.abs().max()) <= 2e-3
