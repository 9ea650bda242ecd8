"""ecq_decode_attention_f16: batch-1 decode attention split over keys, against
a float64 softmax(q.K^T/sqrt(d)).V reference and torch's SDPA, at the head
counts a tensor-parallel rank holds (1-32) and key counts from 1 to 4097;
deterministic replays; and the 7B-shaped decoder with it against SDPA."""
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from ecq_b200 import _lib  # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _attention(q, k, v, splits=None):
    H, T, D = k.shape
    L = _lib.lib()
    if splits is None:
        splits = int(L.ecq_decode_attention_splits(H, T))
    ws = torch.zeros(int(L.ecq_decode_attention_workspace_bytes(H, splits)), dtype=torch.uint8, device="cuda")
    out = torch.empty(H, D, dtype=torch.float16, device="cuda")
    rc = L.ecq_decode_attention_f16(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), H, D, T, T * D,
                                    splits, ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    return out, ws


@pytest.mark.parametrize("H,T", [(4, 2049), (32, 2049), (1, 1), (8, 7), (4, 65), (2, 4097), (1, 8193), (16, 300)])
def test_decode_attention_matches_reference(H, T):
    D = 128
    g = torch.Generator(device="cuda").manual_seed(H * 1000 + T)
    q = torch.randn(H, D, device="cuda", generator=g).half()
    k = torch.randn(H, T, D, device="cuda", generator=g).half()
    v = torch.randn(H, T, D, device="cuda", generator=g).half()
    out, ws = _attention(q, k, v)
    torch.cuda.synchronize()
    assert int(ws[-4 * H:].count_nonzero()) == 0  # counters back at zero
    s = torch.einsum("hd,htd->ht", q.double(), k.double()) / D ** 0.5
    ref = torch.einsum("ht,htd->hd", torch.softmax(s, dim=-1), v.double())
    err = float((out.double() - ref).abs().max() / ref.abs().max())
    assert err <= 2e-3, err
    sdpa = torch.nn.functional.scaled_dot_product_attention(q.view(1, H, 1, D), k.unsqueeze(0), v.unsqueeze(0))
    assert float((out.float() - sdpa.view(H, D).float()).abs().max() / sdpa.float().abs().max()) <= 2e-3
    out2, _ = _attention(q, k, v)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


def test_decode_attention_strided_cache_and_one_split():
    # a cache with one spare slot per head (head stride > keys * D) and a single split
    H, T, D = 4, 100, 128
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(H, D, device="cuda", generator=g).half()
    kc = torch.randn(H, T + 1, D, device="cuda", generator=g).half()
    vc = torch.randn(H, T + 1, D, device="cuda", generator=g).half()
    L = _lib.lib()
    ws = torch.zeros(int(L.ecq_decode_attention_workspace_bytes(H, 1)), dtype=torch.uint8, device="cuda")
    out = torch.empty(H, D, dtype=torch.float16, device="cuda")
    assert L.ecq_decode_attention_f16(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), H, D, T,
                                      (T + 1) * D, 1, ws.data_ptr(), ws.numel(),
                                      torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    s = torch.einsum("hd,htd->ht", q.double(), kc[:, :T].double()) / D ** 0.5
    ref = torch.einsum("ht,htd->hd", torch.softmax(s, dim=-1), vc[:, :T].double())
    assert float((out.double() - ref).abs().max() / ref.abs().max()) <= 2e-3
    assert L.ecq_decode_attention_f16(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), H, 64, T,
                                      (T + 1) * D, 1, ws.data_ptr(), ws.numel(), 0) == -8  # head_dim 64


def test_decoder_with_ecq_attention_matches_sdpa():
    from ecq_b200.model import Llama7BConfig, Llama7BDecoder

    cfg = Llama7BConfig(layers=2, hidden=512, heads=4, head_dim=128, mlp=1024, vocab=1000, kv_len=64)
    a = Llama7BDecoder(cfg, tp=1, seed=7, attention="ecq")
    b = Llama7BDecoder(cfg, tp=1, seed=7, attention="sdpa")
    tok = torch.tensor([11], device="cuda")
    la = a.step_logits(tok).float()
    lb = b.step_logits(tok).float()
    torch.cuda.synchronize()
    a.check()
    assert float((la - lb).abs().max() / lb.abs().max()) <= 1e-2
    assert int(torch.argmax(la)) == int(torch.argmax(lb))
