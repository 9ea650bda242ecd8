"""Tensor-parallel Llama-7B-shaped decode step on rANS-coded weights.

A synthetic Llama-7B (32 layers, hidden 4096, 32 heads x 128, SwiGLU MLP
11008, vocab 32000) whose linear weights are fp16 Student-t(4) * 0.02,
quantised symmetrically per group of 128 (absmax/7, zero-point 8) and
rANS-coded per matrix (one table per matrix, 8-row tiles). Every linear layer
runs the fused decode + dequant + GEMV kernel; the glue (RMSNorm, rotary
embedding, attention over a 2048-token fp16 KV cache, SwiGLU, residuals) is
PyTorch. The reference's model structure is experiments/real_model_test.py:18-113.

Tensor parallelism (one process per GPU, NCCL over NVLink):
  * q/k/v, gate/up and lm_head are column-parallel: each rank owns a range of
    8-row slabs (whole heads for q/k/v);
  * o_proj and down_proj are row-parallel: each rank owns a range of K-tiles
    and the partial outputs are summed with one all-reduce per layer;
  * the gate/up row split follows down_proj's K-tile split, so the MLP needs
    no re-sharding; lm_head logits are all-gathered.
Every matrix is encoded once with its global table and ranks take tile
subsets (codec.slice_matrix), so one encoding serves TP = 1/2/4/8.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

from .codec import RANSTable, encode_matrix, slice_matrix, split_even, choose_tile_cols
from .device import DeviceMatrix
from .ops import rans_gemv

GROUP = 128


@dataclass
class Llama7BConfig:
    layers: int = 32
    hidden: int = 4096
    heads: int = 32
    head_dim: int = 128
    mlp: int = 11008
    vocab: int = 32000
    kv_len: int = 2048
    rope_theta: float = 10000.0
    eps: float = 1e-5


def quantized_student_t(M: int, K: int, seed: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """fp16 Student-t(nu=4) * 0.02 weights, quantised per group of 128 with
    scale = absmax/7 and zero-point 8. Returns (symbols uint8 [M,K], scales fp16
    [M, K/128]) on `device`."""
    g = torch.Generator(device=device).manual_seed(seed)
    # Student-t(4) = N(0,1) / sqrt(chi2_4 / 4), chi2_4 = -2 log(U1 U2)
    z = torch.randn(M, K, generator=g, device=device, dtype=torch.float32)
    u = torch.rand(2, M, K, generator=g, device=device, dtype=torch.float32).clamp_min_(1e-12)
    chi2 = -2.0 * torch.log(u[0] * u[1])
    w = (z / torch.sqrt(chi2 / 4.0) * 0.02).to(torch.float16).float()
    del z, u, chi2
    wg = w.view(M, K // GROUP, GROUP)
    scale = (wg.abs().amax(dim=2) / 7.0).to(torch.float16)
    sc = scale.float()
    safe = torch.where(sc == 0, torch.ones_like(sc), sc)
    q = torch.clamp(torch.round(wg / safe[:, :, None]) + 8, 0, 15).to(torch.uint8).view(M, K)
    return q, scale


class ShardedLinear:
    """One rank's shard of a rANS-coded linear layer."""

    def __init__(self, matrix: DeviceMatrix, scales: torch.Tensor):
        self.m = matrix
        self.scales = scales

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return rans_gemv(x, self.m, self.scales)


def _encode_shard(q_full: torch.Tensor, sc_full: torch.Tensor, slabs: tuple[int, int], ktiles: tuple[int, int] | None,
                  tile_cols: int, device) -> ShardedLinear:
    M, K = q_full.shape
    counts = torch.bincount(q_full.reshape(-1), minlength=16).cpu().numpy()
    table = RANSTable.from_counts(counts)
    nk = K // tile_cols
    k0, k1 = ktiles if ktiles is not None else (0, nk)
    s0, s1 = slabs
    r0, r1 = s0 * 8, min(s1 * 8, M)
    c0, c1 = k0 * tile_cols, k1 * tile_cols
    block = q_full[r0:r1, c0:c1].contiguous().cpu().numpy()
    enc = encode_matrix(block, table, tile_cols=tile_cols, group_size=GROUP)
    m = DeviceMatrix.from_encoded(enc, group_size=GROUP, device=device)
    scales = sc_full[r0:r1, c0 // GROUP:c1 // GROUP].contiguous().to(device)
    return ShardedLinear(m, scales)


class Llama7BDecoder:
    """The decode step of a synthetic Llama-7B on rANS-coded weights, for one
    rank of a tensor-parallel group (tp = world size, rank = this rank)."""

    def __init__(self, cfg: Llama7BConfig | None = None, device=None, tp: int = 1, rank: int = 0, seed: int = 3,
                 group=None):
        self.cfg = cfg = cfg or Llama7BConfig()
        self.dev = torch.device(device or "cuda")
        self.tp, self.rank, self.group = tp, rank, group
        H, D = cfg.hidden, cfg.head_dim
        if cfg.heads % tp:
            raise ValueError("heads must divide evenly over the TP ranks")
        self.local_heads = cfg.heads // tp
        head_slabs = split_even(cfg.heads * D // 8, tp)[rank]  # whole heads: 16 slabs each
        tc_h = choose_tile_cols(H, GROUP)
        tc_m = choose_tile_cols(cfg.mlp, GROUP)
        kt_o = split_even(H // tc_h, tp)[rank]             # o_proj K-tiles (heads)
        kt_d = split_even(cfg.mlp // tc_m, tp)[rank]       # down_proj K-tiles
        mlp_slabs = (kt_d[0] * tc_m // 8, kt_d[1] * tc_m // 8)
        vocab_slabs = split_even((cfg.vocab + 7) // 8, tp)[rank]
        self.mlp_rows = ((mlp_slabs[0] * 8), (mlp_slabs[1] * 8))
        self.vocab_rows = (vocab_slabs[0] * 8, min(vocab_slabs[1] * 8, cfg.vocab))
        if (kt_o[1] - kt_o[0]) * tc_h != self.local_heads * D:
            raise ValueError("o_proj K-tiles do not line up with this rank's heads")
        self.compressed_bytes = 0
        self.symbols = 0
        self.seed = seed
        s = seed
        self.layers = []
        for li in range(cfg.layers):
            lw = {}
            for name, (M, K) in (("q", (H, H)), ("k", (H, H)), ("v", (H, H)), ("o", (H, H)),
                                 ("gate", (cfg.mlp, H)), ("up", (cfg.mlp, H)), ("down", (H, cfg.mlp))):
                q, sc = quantized_student_t(M, K, seed=s, device=self.dev)
                s += 1
                if name in ("q", "k", "v"):
                    lw[name] = _encode_shard(q, sc, head_slabs, None, tc_h, self.dev)
                elif name == "o":
                    lw[name] = _encode_shard(q, sc, (0, H // 8), kt_o, tc_h, self.dev)
                elif name in ("gate", "up"):
                    lw[name] = _encode_shard(q, sc, mlp_slabs, None, tc_h, self.dev)
                else:
                    lw[name] = _encode_shard(q, sc, (0, H // 8), kt_d, tc_m, self.dev)
                self.compressed_bytes += lw[name].m.compressed_bytes
                self.symbols += lw[name].m.rows * lw[name].m.cols
                del q, sc
            lw["ln1"] = torch.ones(H, device=self.dev, dtype=torch.float16)
            lw["ln2"] = torch.ones(H, device=self.dev, dtype=torch.float16)
            self.layers.append(lw)
        q, sc = quantized_student_t(cfg.vocab, H, seed=s, device=self.dev)
        self.lm_head = _encode_shard(q, sc, vocab_slabs, None, tc_h, self.dev)
        self.compressed_bytes += self.lm_head.m.compressed_bytes
        self.symbols += self.lm_head.m.rows * self.lm_head.m.cols
        del q, sc
        g = torch.Generator(device=self.dev).manual_seed(seed + 1000)
        self.embed = (torch.randn(cfg.vocab, H, generator=g, device=self.dev) * 0.02).to(torch.float16)
        self.norm = torch.ones(H, device=self.dev, dtype=torch.float16)
        # 2048-token KV cache of random fp16 values (+1 slot for the new token)
        shape = (cfg.layers, 2, self.local_heads, cfg.kv_len + 1, D)
        self.kv = torch.randn(shape, generator=g, device=self.dev, dtype=torch.float16)
        pos = cfg.kv_len
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, D, 2, device=self.dev, dtype=torch.float32) / D))
        ang = pos * inv
        self.cos = torch.cos(ang).to(torch.float16)
        self.sin = torch.sin(ang).to(torch.float16)
        self.vocab_sizes = [min(hi * 8, cfg.vocab) - lo * 8 for lo, hi in split_even((cfg.vocab + 7) // 8, tp)]
        self.logits = torch.empty(tp, max(self.vocab_sizes), device=self.dev, dtype=torch.float16)

    # -- glue ------------------------------------------------------------------
    def _rms(self, h: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        hf = h.float()
        return (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + self.cfg.eps)).to(torch.float16) * w

    def _rope(self, t: torch.Tensor) -> torch.Tensor:
        a, b = t[..., 0::2], t[..., 1::2]
        return torch.stack((a * self.cos - b * self.sin, a * self.sin + b * self.cos), dim=-1).flatten(-2)

    def _all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.tp > 1:
            dist.all_reduce(t, group=self.group)
        return t

    def step(self, token: torch.Tensor) -> torch.Tensor:
        """One batch-1 decode step: token id (int64 [1], device) -> next token id."""
        return torch.argmax(self.step_logits(token).float()).reshape(1)

    def step_logits(self, token: torch.Tensor) -> torch.Tensor:
        """One batch-1 decode step returning the full fp16 logits [vocab]."""
        cfg = self.cfg
        D, nh = cfg.head_dim, self.local_heads
        h = self.embed[token].reshape(1, cfg.hidden)
        for li, lw in enumerate(self.layers):
            a = self._rms(h, lw["ln1"])
            q = self._rope(lw["q"](a).view(nh, 1, D))
            k = self._rope(lw["k"](a).view(nh, 1, D))
            v = lw["v"](a).view(nh, 1, D)
            self.kv[li, 0, :, cfg.kv_len:cfg.kv_len + 1].copy_(k)
            self.kv[li, 1, :, cfg.kv_len:cfg.kv_len + 1].copy_(v)
            att = torch.nn.functional.scaled_dot_product_attention(
                q.unsqueeze(0), self.kv[li, 0].unsqueeze(0), self.kv[li, 1].unsqueeze(0))
            o = self._all_reduce(lw["o"](att.reshape(1, nh * D)))
            h = h + o
            a = self._rms(h, lw["ln2"])
            m = torch.nn.functional.silu(lw["gate"](a)) * lw["up"](a)
            d = self._all_reduce(lw["down"](m))
            h = h + d
        logits = self.lm_head(self._rms(h, self.norm)).reshape(-1)
        if self.tp > 1:
            local = torch.full((self.logits.shape[1],), -65504.0, device=self.dev, dtype=torch.float16)
            local[: logits.numel()].copy_(logits)
            dist.all_gather_into_tensor(self.logits.view(-1), local, group=self.group)
            return torch.cat([self.logits[i, : self.vocab_sizes[i]] for i in range(self.tp)])
        return logits

    def check(self) -> None:
        for lw in self.layers:
            for k in ("q", "k", "v", "o", "gate", "up", "down"):
                lw[k].m.check()
        self.lm_head.m.check()


def tp_partition(cfg: Llama7BConfig, tp: int) -> list[dict]:
    """The per-rank shard plan (row slabs / K-tiles) of every matrix kind."""
    tc_h = choose_tile_cols(cfg.hidden, GROUP)
    tc_m = choose_tile_cols(cfg.mlp, GROUP)
    plans = []
    for r in range(tp):
        kt_d = split_even(cfg.mlp // tc_m, tp)[r]
        plans.append({
            "qkv_slabs": split_even(cfg.heads * cfg.head_dim // 8, tp)[r],
            "o_ktiles": split_even(cfg.hidden // tc_h, tp)[r],
            "mlp_slabs": (kt_d[0] * tc_m // 8, kt_d[1] * tc_m // 8),
            "down_ktiles": kt_d,
            "vocab_slabs": split_even((cfg.vocab + 7) // 8, tp)[r],
        })
    return plans


__all__ = ["Llama7BConfig", "Llama7BDecoder", "tp_partition", "quantized_student_t", "math"]
