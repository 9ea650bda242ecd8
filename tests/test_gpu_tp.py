"""The tensor-parallel exchange over NVLink peer memory (ecq_gemv_tp ->
ecq_tp_add_rmsnorm_f16 / ecq_tp_sum_f16): one rank on one GPU, two ranks on
2 GPUs, and one rank per GPU when 4 or more are visible. Spawned ranks, NCCL
for the handle exchange and the comparison path."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


# hidden 1024 = two 8x512 K-tiles, so o_proj splits over 2 ranks along whole heads
SMALL_TP_CFG = dict(layers=2, hidden=1024, heads=8, head_dim=128, mlp=2048, vocab=1000, kv_len=64)
# hidden 4096 and mlp 4096 = eight 8x512 K-tiles each: TP 4 and TP 8 get whole tiles and heads
WIDE_TP_CFG = dict(layers=1, hidden=4096, heads=32, head_dim=128, mlp=4096, vocab=1000, kv_len=64)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def _worker(rank, world, port, which):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        if which == "exchange":
            _exchange(rank, world, dev)
        elif which == "exchange_large":
            _exchange(rank, world, dev, M=11008, n_max=11008)
        elif which == "decoder_wide":
            _decoder(rank, world, dev, WIDE_TP_CFG)
        else:
            _decoder(rank, world, dev)
    finally:
        torch.cuda.synchronize()
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()


def _exchange(rank, world, dev, M=520, n_max=1024):
    import ecq_b200 as ecq
    from ecq_b200 import synthetic as syn
    from ecq_b200.codec import slice_matrix, split_even
    from ecq_b200.comm import PeerExchange
    from oracle import oracle

    K, g = 512 * max(4, world), 128  # at least one 512-column K-tile per rank
    sym = syn.laplace_symbols(M, K, b=0.5, seed=61)
    sc = syn.group_scales(M, K, g, seed=62)
    enc = ecq.encode_matrix(sym, tile_cols=512, group_size=g)
    kt0, kt1 = split_even(K // 512, world)[rank]
    m = ecq.DeviceMatrix.from_encoded(slice_matrix(enc, 0, (M + 7) // 8, kt0, kt1), group_size=g, device=dev)
    c0, c1 = kt0 * 512, kt1 * 512
    s_loc = torch.from_numpy(np.ascontiguousarray(sc[:, c0 // g:c1 // g])).to(dev)
    w = torch.from_numpy((1.0 + 0.1 * np.random.default_rng(63).standard_normal(M)).astype(np.float16)).to(dev)
    xch = PeerExchange(n_max=n_max, device=dev)
    try:
        for it in range(5):  # several epochs: both buffer halves, flags re-armed
            x = syn.activations(1, K, seed=70 + it)
            h0 = syn.activations(1, M, seed=80 + it)
            h = torch.from_numpy(h0).to(dev).reshape(-1).clone()
            xch.gemv_push(m, torch.from_numpy(np.ascontiguousarray(x[0, c0:c1])).to(dev), s_loc)
            y = xch.add_rmsnorm(h, w, 1e-5)
            torch.cuda.synchronize()
            m.check()
            xch.check()
            d = oracle.dequant_gemv(sym, sc.astype(np.float32), g, x.astype(np.float32))[0]
            h_ref = (h0[0].astype(np.float32) + d.astype(np.float16).astype(np.float32)).astype(np.float16)
            assert _rel(h.cpu().numpy(), h_ref) <= 2e-3, it
            hf = h_ref.astype(np.float32)
            y_ref = (hf / np.sqrt(np.mean(hf * hf) + 1e-5)).astype(np.float16).astype(np.float32) * \
                w.float().cpu().numpy()
            assert _rel(y.float().cpu().numpy(), y_ref) <= 2e-3, it
        for it in range(3):  # the plain all-reduce consumer, continuing the epochs
            x = syn.activations(1, K, seed=90 + it)
            xch.gemv_push(m, torch.from_numpy(np.ascontiguousarray(x[0, c0:c1])).to(dev), s_loc)
            y = xch.sum(M)
            torch.cuda.synchronize()
            m.check()
            xch.check()
            d = oracle.dequant_gemv(sym, sc.astype(np.float32), g, x.astype(np.float32))[0]
            assert y.shape == (M,) and _rel(y.float().cpu().numpy(), d) <= 2e-3, it
    finally:
        xch.close()


def _decoder(rank, world, dev, cfg_kw=SMALL_TP_CFG):
    from ecq_b200.model import Llama7BConfig, Llama7BDecoder

    cfg = Llama7BConfig(**cfg_kw)
    tok = torch.tensor([17], device=dev)
    ref = Llama7BDecoder(cfg, device=dev, tp=1, seed=5)
    l_ref = ref.step_logits(tok).float()
    dec = Llama7BDecoder(cfg, device=dev, tp=world, rank=rank, seed=5, exchange="peer")
    # every TP size draws the same global KV cache and keeps its heads (the
    # last slot holds the new token's K/V, which ref's step has written)
    nh = dec.local_heads
    kv = cfg.kv_len
    assert torch.equal(dec.kv[:, :, :, :kv], ref.kv[:, :, rank * nh:(rank + 1) * nh, :kv])
    try:
        l_peer = dec.step_logits(tok).float()
        dec.use_peer = False
        l_nccl = dec.step_logits(tok).float()
        dec.use_peer = True
        torch.cuda.synchronize()
        dec.check()
        # peer exchange sums fp32 partials, NCCL fp16 partials: close, not equal
        assert _rel(l_peer.cpu().numpy(), l_nccl.cpu().numpy()) <= 2e-3
        assert _rel(l_peer.cpu().numpy(), l_ref.cpu().numpy()) <= 1e-2
        assert _rel(l_nccl.cpu().numpy(), l_ref.cpu().numpy()) <= 1e-2
        # the exchange inside a CUDA graph: the epoch advances on the device
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=s):
                out = dec.step_logits(tok)
            for _ in range(4):
                gr.replay()
            s.synchronize()
        dec.check()
        assert torch.equal(out.float(), l_peer)
        del gr
    finally:
        dec.close()


@pytest.mark.parametrize("which", ["exchange", "exchange_large"])
def test_peer_exchange_one_rank(which):
    """One rank pushing to itself: the fused GEMV's push and both cluster
    consumers (8 CTAs; 520 and 11008 rows) against the oracle over several
    epochs, on one GPU."""
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(1, _free_port(), which), nprocs=1, join=True)


@pytest.mark.parametrize("which", ["exchange", "exchange_large", "decoder"])
def test_peer_exchange_two_gpus(which):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _free_port(), which), nprocs=2, join=True)


@pytest.mark.parametrize("which", ["exchange", "decoder_wide"])
def test_peer_exchange_all_gpus(which):
    """The same checks with one rank per visible GPU (4 or 8 on one box)."""
    n = torch.cuda.device_count()
    if n < 4:
        pytest.skip("needs 4 or more GPUs")
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(n, _free_port(), which), nprocs=n, join=True)
