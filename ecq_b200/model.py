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
Each matrix (q|k|v and gate|up as fused projections sharing one table) is
encoded with its global table and every rank encodes exactly the tiles of its
shard, which are the same tiles whatever the TP size. A layer launches 4
fused GEMVs -- q|k|v with the rotary embedding and the KV-cache store fused
into its epilogue, gate|up (rows interleaved) with SwiGLU fused in -- one
residual add + RMSNorm before each of the two projections that read the
residual stream (with TP > 1 these are the exchange consumers, the
row-parallel sums fused into the GEMV push and the consumer) and attention.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ._lib import check, lib
from .codec import RANSTable, concat_rows, encode_matrix, split_even, choose_tile_cols
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


# A batch-1 GEMV runs its tiles in rounds over the GPU's warp slots (one CTA of
# up to 32 warps per SM), and each round waits on one tile's serial decode of
# tile_cols / 4 symbols per lane plus a fixed per-tile cost. Narrow tiles
# shorten the chain but add tiles (rounds) and per-tile overhead, and compress
# worse. shard_tile_cols picks the width with the least modelled time,
# ceil(tiles / warp slots) * (tile_cols / 4 + TILE_OVERHEAD); on the TP shard
# shapes of the 7B layers and the sweep (1536..22016 rows x 512..11008 columns)
# it picks the fastest measured width or one within 3 % of it.
# Heads per rank up to which "auto" picks the split-key decode attention. It
# measured slower than cuDNN's SDPA at every head count from 2 to 32 (2049
# keys, head_dim 128, CUDA graph of 32 layers: 9.2-19.1 us against 6.6-11.2
# us), so "auto" always picks SDPA.
ECQ_ATTENTION_MAX_HEADS = 0

WARP_SLOTS = 148 * 32
TILE_OVERHEAD = 40


def shard_tile_cols(rows: int, cols: int, group: int = GROUP, warp_slots: int = WARP_SLOTS) -> int:
    """Tile width (512 / 256 / 128 columns) for encoding one [rows, cols]
    shard: of the widths compatible with cols and the group size, the one
    with the least modelled decode time (ties: the widest)."""
    ok = [c for c in (512, 256, 128) if cols % c == 0 and (c % group == 0 if group < c else group % c == 0)]
    if not ok:
        raise ValueError(f"no tile width for {cols} columns, group {group}")
    slabs = (rows + 7) // 8

    def cost(c):
        tiles = slabs * (cols // c)
        return ((tiles + warp_slots - 1) // warp_slots) * (c // 4 + TILE_OVERHEAD)

    return min(ok, key=lambda c: (cost(c), -c))


def _encode_shards(parts, table: RANSTable, tile_cols: int | None, device) -> ShardedLinear:
    """Encode the row blocks `parts` = [(symbols, scales, (r0, r1), (c0, c1)), ...]
    with one shared table and stack them into one packed matrix (tile width
    `tile_cols`, or chosen by shard_tile_cols for the stacked shape)."""
    if tile_cols is None:
        rows = sum(r1 - r0 for _, _, (r0, r1), _ in parts)
        c0, c1 = parts[0][3]
        tile_cols = shard_tile_cols(rows, c1 - c0)
    encs, scs = [], []
    for q_full, sc_full, (r0, r1), (c0, c1) in parts:
        block = q_full[r0:r1, c0:c1].contiguous().cpu().numpy()
        encs.append(encode_matrix(block, table, tile_cols=tile_cols, group_size=GROUP))
        scs.append(sc_full[r0:r1, c0 // GROUP:c1 // GROUP])
    enc = concat_rows(encs) if len(encs) > 1 else encs[0]
    m = DeviceMatrix.from_encoded(enc, group_size=GROUP, device=device)
    return ShardedLinear(m, torch.cat(scs, dim=0).contiguous().to(device))


def _table_of(*mats: torch.Tensor) -> RANSTable:
    counts = sum(torch.bincount(q.reshape(-1), minlength=16) for q in mats)
    return RANSTable.from_counts(counts.cpu().numpy())


class Llama7BDecoder:
    """The decode step of a synthetic Llama-7B on rANS-coded weights, for one
    rank of a tensor-parallel group (tp = world size, rank = this rank)."""

    def __init__(self, cfg: Llama7BConfig | None = None, device=None, tp: int = 1, rank: int = 0, seed: int = 3,
                 group=None, exchange: str = "peer", attention: str = "auto"):
        """exchange (tp > 1): "peer" fuses each row-parallel layer's all-reduce
        into its GEMV and the next add + RMSNorm over NVLink peer memory
        (ecq_b200.comm); "nccl" runs GEMV -> NCCL all-reduce -> add + RMSNorm.
        attention: "ecq" runs libecq's split-key decode attention
        (ecq_decode_attention_f16), "sdpa" torch's scaled_dot_product_attention,
        "auto" the first for at most ECQ_ATTENTION_MAX_HEADS heads per rank
        (where it was measured faster), the second above."""
        self.cfg = cfg = cfg or Llama7BConfig()
        if attention not in ("ecq", "sdpa", "auto"):
            raise ValueError("attention is 'ecq', 'sdpa' or 'auto'")
        if attention == "auto":
            attention = "ecq" if cfg.heads // tp <= ECQ_ATTENTION_MAX_HEADS else "sdpa"
        self.attention = attention
        self.dev = torch.device(device or "cuda")
        self.tp, self.rank, self.group = tp, rank, group
        if exchange not in ("peer", "nccl"):
            raise ValueError("exchange is 'peer' or 'nccl'")
        self.exchange = exchange if tp > 1 else "none"
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
        hr = (head_slabs[0] * 8, head_slabs[1] * 8)
        mr = (mlp_slabs[0] * 8, mlp_slabs[1] * 8)
        for li in range(cfg.layers):
            lw = {}
            W = {}
            for name, (M, K) in (("q", (H, H)), ("k", (H, H)), ("v", (H, H)), ("o", (H, H)),
                                 ("gate", (cfg.mlp, H)), ("up", (cfg.mlp, H)), ("down", (H, cfg.mlp))):
                W[name] = quantized_student_t(M, K, seed=s, device=self.dev)
                s += 1
            t_qkv = _table_of(W["q"][0], W["k"][0], W["v"][0])
            lw["qkv"] = _encode_shards([(W[n][0], W[n][1], hr, (0, H)) for n in ("q", "k", "v")], t_qkv, None,
                                       self.dev)
            lw["o"] = _encode_shards([(W["o"][0], W["o"][1], (0, H), (kt_o[0] * tc_h, kt_o[1] * tc_h))],
                                     _table_of(W["o"][0]), None, self.dev)
            t_gu = _table_of(W["gate"][0], W["up"][0])
            # gate and up rows interleaved (row 2j gate j, 2j + 1 up j), so the
            # GEMV's epilogue finds each pair in one row slab for SwiGLU
            gu_q = torch.stack((W["gate"][0][mr[0]:mr[1]], W["up"][0][mr[0]:mr[1]]), dim=1).reshape(-1, H)
            gu_s = torch.stack((W["gate"][1][mr[0]:mr[1]], W["up"][1][mr[0]:mr[1]]), dim=1).reshape(gu_q.shape[0], -1)
            lw["gate_up"] = _encode_shards([(gu_q, gu_s, (0, gu_q.shape[0]), (0, H))], t_gu, None, self.dev)
            del gu_q, gu_s
            lw["down"] = _encode_shards([(W["down"][0], W["down"][1], (0, H), (kt_d[0] * tc_m, kt_d[1] * tc_m))],
                                        _table_of(W["down"][0]), None, self.dev)
            del W
            for k in ("qkv", "o", "gate_up", "down"):
                self.compressed_bytes += lw[k].m.compressed_bytes
                self.symbols += lw[k].m.rows * lw[k].m.cols
            lw["ln1"] = torch.ones(H, device=self.dev, dtype=torch.float16)
            lw["ln2"] = torch.ones(H, device=self.dev, dtype=torch.float16)
            self.layers.append(lw)
        q, sc = quantized_student_t(cfg.vocab, H, seed=s, device=self.dev)
        vr = (vocab_slabs[0] * 8, min(vocab_slabs[1] * 8, cfg.vocab))
        self.lm_head = _encode_shards([(q, sc, vr, (0, H))], _table_of(q), None, self.dev)
        self.compressed_bytes += self.lm_head.m.compressed_bytes
        self.symbols += self.lm_head.m.rows * self.lm_head.m.cols
        del q, sc
        g = torch.Generator(device=self.dev).manual_seed(seed + 1000)
        self.embed = (torch.randn(cfg.vocab, H, generator=g, device=self.dev) * 0.02).to(torch.float16)
        self.norm = torch.ones(H, device=self.dev, dtype=torch.float16)
        # 2048-token KV cache of random fp16 values (+1 slot for the new token):
        # every layer's cache is drawn for all heads and this rank keeps its
        # heads, so every TP size decodes against the same cache
        shape = (cfg.layers, 2, self.local_heads, cfg.kv_len + 1, D)
        self.kv = torch.empty(shape, device=self.dev, dtype=torch.float16)
        h0 = rank * self.local_heads
        for li in range(cfg.layers):
            full = torch.randn((2, cfg.heads, cfg.kv_len + 1, D), generator=g, device=self.dev, dtype=torch.float16)
            self.kv[li].copy_(full[:, h0:h0 + self.local_heads])
            del full
        pos = cfg.kv_len
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, D, 2, device=self.dev, dtype=torch.float32) / D))
        ang = pos * inv
        self.cos = torch.cos(ang).to(torch.float16)
        self.sin = torch.sin(ang).to(torch.float16)
        self.vocab_sizes = [min(hi * 8, cfg.vocab) - lo * 8 for lo, hi in split_even((cfg.vocab + 7) // 8, tp)]
        self.logits = torch.empty(tp, max(self.vocab_sizes), device=self.dev, dtype=torch.float16)
        self.xch = None
        self._marks = None  # CUDA events of a step_breakdown run
        keys = cfg.kv_len + 1
        self.att_splits = int(lib().ecq_decode_attention_splits(self.local_heads, keys))
        self.att_ws = torch.zeros(int(lib().ecq_decode_attention_workspace_bytes(self.local_heads, self.att_splits)),
                                  dtype=torch.uint8, device=self.dev)
        self.att_out = torch.empty(1, self.local_heads * D, dtype=torch.float16, device=self.dev)
        self.use_peer = True  # with an exchange: False runs the NCCL path instead (same weights)
        if self.exchange == "peer":
            from .comm import PeerExchange

            self.xch = PeerExchange(n_max=H, group=group, device=self.dev)

    # -- glue ------------------------------------------------------------------
    def _add_rms(self, h: torch.Tensor, d: torch.Tensor | None, w: torch.Tensor) -> torch.Tensor:
        """h += d (in place, when d is given); returns rmsnorm(h) * w."""
        y = torch.empty_like(h)
        check(lib().ecq_add_rmsnorm_f16(h.data_ptr(), d.data_ptr() if d is not None else None, w.data_ptr(),
                                        h.data_ptr(), y.data_ptr(), h.shape[0], h.shape[1], self.cfg.eps,
                                        torch.cuda.current_stream(self.dev).cuda_stream), "add_rmsnorm")
        return y

    def _all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.tp > 1:
            dist.all_reduce(t, group=self.group)
        return t

    def step(self, token: torch.Tensor) -> torch.Tensor:
        """One batch-1 decode step: token id (int64 [1], device) -> next token id."""
        return torch.argmax(self.step_logits(token).float()).reshape(1)

    def _mark(self, label: str) -> None:
        """Close the current timed interval under `label` (breakdown runs only)."""
        if self._marks is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(torch.cuda.current_stream(self.dev))
            self._marks.append((label, ev))

    def step_breakdown(self, token: torch.Tensor, sleep_cycles: int = 20_000_000) -> dict:
        """Device time of one decode step split by kernel kind: CUDA events
        between consecutive launches of an eager step. A device-side sleep is
        queued first, so that the host has queued the whole step before the
        GPU reaches it and host launch gaps do not enter the intervals.
        Events between launches also stop consecutive kernels from
        overlapping their prologues, so the parts add up to a little more
        than a CUDA-graph step. Returns {kind: microseconds per step}."""
        torch.cuda.synchronize(self.dev)
        self._marks = []
        try:
            torch.cuda._sleep(int(sleep_cycles))
            self._mark("start")
            self.step_logits(token)
            torch.cuda.synchronize(self.dev)
            out: dict = {}
            for (_, a), (label, b) in zip(self._marks[:-1], self._marks[1:]):
                out[label] = out.get(label, 0.0) + a.elapsed_time(b) * 1e3
        finally:
            self._marks = None
        out["total"] = sum(out.values())
        return {k: round(v, 1) for k, v in out.items()}

    def step_logits(self, token: torch.Tensor) -> torch.Tensor:
        """One batch-1 decode step returning the full fp16 logits [vocab]."""
        cfg = self.cfg
        D, nh = cfg.head_dim, self.local_heads
        L = nh * D
        mk = self._mark
        h = self.embed[token].reshape(1, cfg.hidden).clone()
        mk("embed")
        d = None
        peer = self.xch is not None and self.use_peer
        pending = False  # the residual delta sits in the peer exchange (not in d)
        nvtx = torch.cuda.nvtx
        for li, lw in enumerate(self.layers):
            nvtx.range_push(f"layer {li}")  # one NVTX range per layer for timeline profilers
            if pending:
                a = self.xch.add_rmsnorm(h, lw["ln1"], cfg.eps)
                mk("exchange consumer: sum + add + rmsnorm")
            else:
                a = self._add_rms(h, d, lw["ln1"])
                mk("add + rmsnorm")
            kslot = self.kv[li, 0, :, cfg.kv_len]
            vslot = self.kv[li, 1, :, cfg.kv_len]
            # [1, 3L]: q | k | v, q and k rotated, k and v stored into the cache slot
            qkv = lw["qkv"].m.gemv_rope_kv(a, lw["qkv"].scales, self.cos, self.sin, kslot, vslot, D,
                                           (cfg.kv_len + 1) * D)
            mk("gemv q|k|v + rope + kv write")
            if self.attention == "ecq":
                att = self.att_out
                check(lib().ecq_decode_attention_f16(qkv.data_ptr(), self.kv[li, 0].data_ptr(),
                                                     self.kv[li, 1].data_ptr(), att.data_ptr(), nh, D,
                                                     cfg.kv_len + 1, (cfg.kv_len + 1) * D, self.att_splits,
                                                     self.att_ws.data_ptr(), self.att_ws.numel(),
                                                     torch.cuda.current_stream(self.dev).cuda_stream),
                      "decode attention")
                mk("attention (ecq split-key)")
            else:
                q = qkv[:, :L].reshape(1, nh, 1, D)
                att = torch.nn.functional.scaled_dot_product_attention(q, self.kv[li, 0].unsqueeze(0),
                                                                       self.kv[li, 1].unsqueeze(0))
                mk("attention (sdpa)")
            if peer:
                self.xch.gemv_push(lw["o"].m, att.reshape(1, L).contiguous(), lw["o"].scales)
                mk("gemv o + push")
                a = self.xch.add_rmsnorm(h, lw["ln2"], cfg.eps)
                mk("exchange consumer: sum + add + rmsnorm")
            else:
                o = lw["o"](att.reshape(1, L))
                mk("gemv o")
                if self.tp > 1:
                    o = self._all_reduce(o)
                    mk("nccl all-reduce")
                a = self._add_rms(h, o, lw["ln2"])
                mk("add + rmsnorm")
            m = lw["gate_up"].m.gemv_silu_mul(a, lw["gate_up"].scales)  # [1, F] = silu(gate) * up
            mk("gemv gate|up + silu * mul")
            if peer:
                self.xch.gemv_push(lw["down"].m, m, lw["down"].scales)
                mk("gemv down + push")
                pending = True
            else:
                d = lw["down"](m)
                mk("gemv down")
                if self.tp > 1:
                    d = self._all_reduce(d)
                    mk("nccl all-reduce")
            nvtx.range_pop()
        if pending:
            a = self.xch.add_rmsnorm(h, self.norm, cfg.eps)
            mk("exchange consumer: sum + add + rmsnorm")
        else:
            a = self._add_rms(h, d, self.norm)
            mk("add + rmsnorm")
        logits = self.lm_head(a).reshape(-1)
        mk("gemv lm_head")
        if self.tp > 1:
            local = torch.full((self.logits.shape[1],), -65504.0, device=self.dev, dtype=torch.float16)
            local[: logits.numel()].copy_(logits)
            dist.all_gather_into_tensor(self.logits.view(-1), local, group=self.group)
            out = torch.cat([self.logits[i, : self.vocab_sizes[i]] for i in range(self.tp)])
            mk("logits all-gather")
            return out
        return logits

    def check(self) -> None:
        for lw in self.layers:
            for k in ("qkv", "o", "gate_up", "down"):
                lw[k].m.check()
        self.lm_head.m.check()
        if self.xch is not None:
            self.xch.check()

    def close(self) -> None:
        """Release the peer exchange (collective over the TP group)."""
        if self.xch is not None:
            self.xch.close()
            self.xch = None


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


__all__ = ["Llama7BConfig", "Llama7BDecoder", "tp_partition", "shard_tile_cols", "quantized_student_t"]
