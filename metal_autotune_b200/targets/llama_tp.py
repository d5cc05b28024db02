"""Llama-3-8B (MLX-affine 8-bit, group 64) prefill forward, tensor-parallel.

The target is the reference's Llama model (models/llama8b.py:4-7, mlx-lm
llama at 8 bits): batch 8 x 2048 prompt tokens, random-initialised. Per layer:
rms_norm -> q/k/v qmm -> rope(theta 5e5) -> causal GQA SDPA -> o qmm ->
+residual -> rms_norm -> gate/up qmm + swiglu -> down qmm -> +residual; final
rms_norm; lm_head on each sequence's last position. Every op is a libmt.so
entry point (rope reads the token-major q/k projections and writes them
head-major, the transpose MLX applies before its rope in mlx-lm's llama);
the only torch work is the collectives.

Tensor parallel over `tp` shards:
  - q/k/v and gate/up are column-parallel: shard r holds output rows
    [r*N/tp, (r+1)*N/tp), i.e. whole heads (32/tp query, 8/tp kv heads) and
    whole FFN columns;
  - o and down are row-parallel: shard r holds input columns
    [r*K/tp, (r+1)*K/tp) as whole g64 groups (packed words and scale/bias
    columns sliced alike; 4096/8 = 512 and 14336/8 = 1792 are multiples of
    64), so each shard's output is a partial sum over its slice of K;
  - the partials are summed over the shards (one all-reduce, bf16, per
    row-parallel projection: 2 per layer), then added to the residual with
    the next RMSNorm fused (mt_add_rms_norm);
  - lm_head is vocab-parallel: each shard computes its vocab rows for the
    last positions, and the logits are gathered.
Every shard of every tp degree is a slice of the same seeded model, so the
outputs at any tp agree up to the order of the partial sums.

Shards run either one per process (`ProcessGroupComm`, NCCL on the GPU box)
or all in one process (`LocalComm`, the sum taken in shard order), which
lets one GPU check tp > 1 against tp = 1. With one shard per process the
forward runs as two software-pipelined micro-batches, each micro-batch's
all-reduce overlapping the other's next block of compute
(`_forward_overlapped`; `overlap=False` gives the serial forward).
"""
from __future__ import annotations

import functools
import math
from dataclasses import dataclass

import torch

from .. import lib, workload


@dataclass(frozen=True)
class LlamaConfig:
    hidden: int = 4096
    layers: int = 32
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    vocab: int = 128256
    rope_theta: float = 5e5
    eps: float = 1e-5
    group: int = 64
    bits: int = 8


LLAMA3_8B = LlamaConfig()
TINY = LlamaConfig(hidden=512, layers=2, heads=4, kv_heads=2, head_dim=128, ffn=1024, vocab=1024)


# ------------------------------------------------------------------ sharding
def shard_rows(qset, r: int, tp: int):
    """Column-parallel shard r of a quantised projection: output rows
    [r*N/tp, (r+1)*N/tp) of (packed weights, scales, biases)."""
    wq, s, b = qset
    N = wq.shape[0]
    if N % tp:
        raise ValueError(f"N={N} does not split over tp={tp}")
    n = N // tp
    return tuple(t[r * n:(r + 1) * n].contiguous() for t in (wq, s, b))


def shard_cols(qset, r: int, tp: int, group: int, bits: int):
    """Row-parallel shard r of a quantised projection: input columns
    [r*K/tp, (r+1)*K/tp), kept as whole quantisation groups so the slice of
    the packed words and of the scale/bias columns dequantises to exactly the
    slice of the full weight."""
    wq, s, b = qset
    K = s.shape[1] * group
    if K % (tp * group):
        raise ValueError(f"K={K} does not split over tp={tp} in whole groups of {group}")
    k = K // tp
    per = 32 // bits
    w = wq[:, r * k // per:(r + 1) * k // per].contiguous()
    g0, g1 = r * k // group, (r + 1) * k // group
    return w, s[:, g0:g1].contiguous(), b[:, g0:g1].contiguous()


# ------------------------------------------------------------------ collectives
class LocalComm:
    """Every shard in this process: the all-reduce is a bf16 sum in shard
    order, the gather a concatenation along the last axis."""

    def all_reduce(self, parts):
        return functools.reduce(torch.add, parts)

    def all_gather(self, parts):
        return torch.cat(parts, dim=-1)


class ProcessGroupComm:
    """One shard per rank of the default process group (NCCL on GPUs)."""

    def __init__(self):
        import torch.distributed as dist
        self.dist = dist
        self.world = dist.get_world_size()

    def all_reduce(self, parts):
        (p,) = parts
        self.dist.all_reduce(p)
        return p

    def all_reduce_async(self, p):
        """Start an in-place sum of p over the ranks; returns the handle whose
        wait() makes the current stream wait for the sum (the host does not block)."""
        return self.dist.all_reduce(p, async_op=True)

    def all_gather(self, parts):
        (p,) = parts
        outs = [torch.empty_like(p) for _ in range(self.world)]
        self.dist.all_gather(outs, p.contiguous())
        return torch.cat(outs, dim=-1)


# ------------------------------------------------------------------ model
class ShardLayer:
    def __init__(self, q, k, v, o, gate, up, down):
        self.qkv = (q, k, v)
        self.o, self.gate, self.up, self.down = o, gate, up, down


class Shard:
    def __init__(self, layers: list[ShardLayer], lm_head):
        self.layers = layers
        self.lm_head = lm_head


def _gen(seed: int, layer: int, j: int, device):
    return torch.Generator(device=device).manual_seed(seed * 1_000_003 + layer * 16 + j)


class LlamaTP:
    """Shards `ranks` of a tp-way split of one seeded Llama model.

    Weights are N(0, 0.02) quantised to MLX affine (cfg.group, cfg.bits), norms
    are 1, the embedding table is replicated on every shard holder, lm_head
    is split by vocab rows."""

    def __init__(self, cfg: LlamaConfig, tp: int, ranks, comm, seed: int = 0, device="cuda",
                 dtype=torch.bfloat16, overlap: bool = True):
        self.cfg, self.tp, self.ranks, self.comm = cfg, tp, list(ranks), comm
        self.overlap = overlap
        self.dtype, self.device = dtype, device
        if cfg.heads % tp or cfg.kv_heads % tp:
            raise ValueError(f"{cfg.heads}/{cfg.kv_heads} heads do not split over tp={tp}")
        self.hq, self.hkv = cfg.heads // tp, cfg.kv_heads // tp
        D = cfg.head_dim

        def full(n, k, layer, j):
            return workload.random_quantized(n, k, group=cfg.group, bits=cfg.bits, dtype=dtype,
                                             generator=_gen(seed, layer, j, device), device=device)

        per_rank = {r: [] for r in self.ranks}
        shapes = [(cfg.heads * D, cfg.hidden), (cfg.kv_heads * D, cfg.hidden), (cfg.kv_heads * D, cfg.hidden),
                  (cfg.hidden, cfg.heads * D), (cfg.ffn, cfg.hidden), (cfg.ffn, cfg.hidden), (cfg.hidden, cfg.ffn)]
        for li in range(cfg.layers):
            sets = {r: [] for r in self.ranks}
            for j, (n, k) in enumerate(shapes):
                w = full(n, k, li, j)
                for r in self.ranks:
                    row_parallel = j in (3, 6)
                    sets[r].append(shard_cols(w, r, tp, cfg.group, cfg.bits) if row_parallel
                                   else shard_rows(w, r, tp))
                del w
            for r in self.ranks:
                per_rank[r].append(ShardLayer(*sets[r]))
        self.embed = full(cfg.vocab, cfg.hidden, cfg.layers, 0)
        head = full(cfg.vocab, cfg.hidden, cfg.layers, 1)  # Llama-3 does not tie lm_head to the embedding
        self.shards = [Shard(per_rank[r], shard_rows(head, r, tp)) for r in self.ranks]
        del head
        ones = torch.ones(cfg.hidden, dtype=dtype, device=device)
        self.attn_norm = [ones] * cfg.layers
        self.mlp_norm = [ones] * cfg.layers
        self.final_norm = ones

    # one shard's attention block: rows of x -> its partial of o_proj
    def _attn(self, sl: ShardLayer, xn, B, L):
        cfg, D = self.cfg, self.cfg.head_dim
        q, k, v = lib.quantized_matmul_multi(xn, list(sl.qkv), group_size=cfg.group, bits=cfg.bits)
        # rope reads the token-major projections and writes head-major q and k
        qr = lib.rope_bhld(q.view(B, L, self.hq, D).transpose(1, 2), D, base=cfg.rope_theta)
        kr = lib.rope_bhld(k.view(B, L, self.hkv, D).transpose(1, 2), D, base=cfg.rope_theta)
        vh = v.view(B, L, self.hkv, D).transpose(1, 2)
        o = lib.sdpa(qr, kr, vh, scale=1.0 / math.sqrt(D), causal=True, out_layout="blhd")
        return lib.quantized_matmul(o.view(B * L, self.hq * D), *sl.o, group_size=cfg.group, bits=cfg.bits)

    def _mlp(self, sl: ShardLayer, xn):
        cfg = self.cfg
        act = lib.quantized_matmul_swiglu(xn, *sl.gate, *sl.up, group_size=cfg.group, bits=cfg.bits)
        return lib.quantized_matmul(act, *sl.down, group_size=cfg.group, bits=cfg.bits)

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        """tokens int32 [B, L] -> logits [B, vocab] of each sequence's last position."""
        cfg = self.cfg
        B, L = tokens.shape
        if self.overlap and hasattr(self.comm, "all_reduce_async") and len(self.shards) == 1 and B >= 2 and B % 2 == 0:
            return self._forward_overlapped(tokens)
        h = lib.quantized_embedding(tokens.reshape(-1), *self.embed, group_size=cfg.group, bits=cfg.bits,
                                    dtype=self.dtype)
        xn = lib.rms_norm(h, self.attn_norm[0], cfg.eps)
        for li in range(cfg.layers):
            o = self.comm.all_reduce([self._attn(s.layers[li], xn, B, L) for s in self.shards])
            h, xn = lib.add_rms_norm(o, h, self.mlp_norm[li], cfg.eps)
            d = self.comm.all_reduce([self._mlp(s.layers[li], xn) for s in self.shards])
            nxt = self.attn_norm[li + 1] if li + 1 < cfg.layers else self.final_norm
            h, xn = lib.add_rms_norm(d, h, nxt, cfg.eps)
        last = xn.view(B, L, cfg.hidden)[:, -1].contiguous()
        parts = [lib.quantized_matmul(last, *s.lm_head, group_size=cfg.group, bits=cfg.bits) for s in self.shards]
        return self.comm.all_gather(parts)

    def _forward_overlapped(self, tokens: torch.Tensor) -> torch.Tensor:
        """The same forward in two micro-batches (the first and the second half
        of the sequences; attention never mixes sequences), software-pipelined
        on one compute stream: each micro-batch's all-reduce is started
        asynchronously (NCCL, its own stream) and waited for only after the
        other micro-batch's next attention or MLP block has been issued, so
        every all-reduce runs beside a block of compute. The sums are the same
        per micro-batch; only the partition of the projections' launches
        changes (reordered fp32 partial sums, within the tolerance of the
        unsplit forward)."""
        cfg = self.cfg
        B, L = tokens.shape
        sh = self.shards[0]
        comm = self.comm
        h = lib.quantized_embedding(tokens.reshape(-1), *self.embed, group_size=cfg.group, bits=cfg.bits,
                                    dtype=self.dtype)
        xn = lib.rms_norm(h, self.attn_norm[0], cfg.eps)
        half = (B // 2) * L
        hs, xns = [h[:half], h[half:]], [xn[:half], xn[half:]]
        pend: list = [None, None]
        for li in range(cfg.layers):
            sl = sh.layers[li]
            for m in (0, 1):
                if pend[m] is not None:
                    work, d = pend[m]
                    work.wait()
                    hs[m], xns[m] = lib.add_rms_norm(d, hs[m], self.attn_norm[li], cfg.eps)
                o = self._attn(sl, xns[m], B // 2, L)
                pend[m] = (comm.all_reduce_async(o), o)
            for m in (0, 1):
                work, o = pend[m]
                work.wait()
                hs[m], xns[m] = lib.add_rms_norm(o, hs[m], self.mlp_norm[li], cfg.eps)
                d = self._mlp(sl, xns[m])
                pend[m] = (comm.all_reduce_async(d), d)
        for m in (0, 1):
            work, d = pend[m]
            work.wait()
            hs[m], xns[m] = lib.add_rms_norm(d, hs[m], self.final_norm, cfg.eps)
        last = torch.cat([x.view(B // 2, L, cfg.hidden)[:, -1] for x in xns]).contiguous()
        part = lib.quantized_matmul(last, *sh.lm_head, group_size=cfg.group, bits=cfg.bits)
        return comm.all_gather([part])

    __call__ = forward


def forward_flops(cfg: LlamaConfig, B: int, L: int) -> float:
    """Algorithmic FLOPs of one prefill forward: projections 2*T*N*K,
    causal attention 2 * 2*B*H*D * L(L+1)/2, lm_head on B rows."""
    T = B * L
    D = cfg.head_dim
    proj = (cfg.heads * D + 2 * cfg.kv_heads * D) * cfg.hidden + cfg.hidden * cfg.heads * D \
        + 3 * cfg.ffn * cfg.hidden
    attn = 2 * 2 * B * cfg.heads * D * (L * (L + 1) / 2)
    return cfg.layers * (2 * T * proj + attn) + 2 * B * cfg.vocab * cfg.hidden
