"""The Llama-shaped decode step (model.py) on a small configuration, TP = 1:
logits from the rANS-coded fused GEMVs against the same step computed with
plain fp32 matmuls on the dequantised weights."""
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from ecq_b200.model import Llama7BConfig, Llama7BDecoder, quantized_student_t  # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _dequant(q, sc):
    return (q.float() - 8.0) * sc.float().repeat_interleave(128, dim=1)


def _rms(h, w, eps=1e-5):
    hf = h.float()
    return (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + eps)).to(torch.float16) * w


def _rope(t, cos, sin):
    a, b = t[..., 0::2].float(), t[..., 1::2].float()
    c, s = cos.float(), sin.float()
    return torch.stack((a * c - b * s, a * s + b * c), dim=-1).flatten(-2).to(torch.float16)


def test_small_decoder_matches_fp32_reference():
    cfg = Llama7BConfig(layers=2, hidden=512, heads=4, head_dim=128, mlp=1024, vocab=1000, kv_len=64)
    dec = Llama7BDecoder(cfg, tp=1, seed=5)
    kv0 = dec.kv.clone()
    tok = torch.tensor([17], device="cuda")
    logits = dec.step_logits(tok).float()
    torch.cuda.synchronize()
    dec.check()
    # reference: same glue, fp32 matmuls on dequantised weights
    s = dec.seed
    W = []
    for _ in range(cfg.layers):
        lw = {}
        for name, (M, K) in (("q", (512, 512)), ("k", (512, 512)), ("v", (512, 512)), ("o", (512, 512)),
                             ("gate", (1024, 512)), ("up", (1024, 512)), ("down", (512, 1024))):
            q, sc = quantized_student_t(M, K, seed=s, device="cuda")
            s += 1
            lw[name] = _dequant(q, sc)
        W.append(lw)
    q, sc = quantized_student_t(cfg.vocab, 512, seed=s, device="cuda")
    Wl = _dequant(q, sc)
    lin = lambda w, x: (x.float() @ w.t()).to(torch.float16)
    kv = kv0
    h = dec.embed[tok].reshape(1, 512)
    for li, lw in enumerate(W):
        a = _rms(h, torch.ones(512, device="cuda", dtype=torch.float16))
        qh = _rope(lin(lw["q"], a).view(4, 1, 128), dec.cos, dec.sin)
        kh = _rope(lin(lw["k"], a).view(4, 1, 128), dec.cos, dec.sin)
        vh = lin(lw["v"], a).view(4, 1, 128)
        kv[li, 0, :, 64:65].copy_(kh)
        kv[li, 1, :, 64:65].copy_(vh)
        att = torch.nn.functional.scaled_dot_product_attention(qh.unsqueeze(0), kv[li, 0].unsqueeze(0),
                                                               kv[li, 1].unsqueeze(0))
        h = h + lin(lw["o"], att.reshape(1, 512))
        a = _rms(h, torch.ones(512, device="cuda", dtype=torch.float16))
        m = torch.nn.functional.silu(lin(lw["gate"], a)) * lin(lw["up"], a)
        h = h + lin(lw["down"], m)
    ref = lin(Wl, _rms(h, dec.norm)).reshape(-1).float()
    err = float((logits - ref).abs().max() / ref.abs().max())
    assert err < 1e-2, err
    assert int(torch.argmax(logits)) == int(torch.argmax(ref))


def test_decoder_step_in_cuda_graph():
    cfg = Llama7BConfig(layers=2, hidden=512, heads=4, head_dim=128, mlp=1024, vocab=1000, kv_len=64)
    dec = Llama7BDecoder(cfg, tp=1, seed=6)
    tok = torch.tensor([3], device="cuda")
    eager = dec.step(tok)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        dec.step(tok)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            out = dec.step(tok)
    g.replay()
    torch.cuda.synchronize()
    dec.check()
    assert int(out) == int(eager)
