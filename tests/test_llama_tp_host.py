"""Host-side checks of the Llama tensor-parallel split (no GPU).

The shards of a quantised projection dequantise to exact slices of the full
weight, and a column-parallel -> row-parallel pair (the shape of both the
attention and the MLP block) summed over two gloo ranks reproduces the
unsharded product: the partitioning the B200 path runs with NCCL."""
from __future__ import annotations

import pytest
import torch
import torch.multiprocessing as mp

from metal_autotune_b200 import workload
from metal_autotune_b200.targets import llama_tp


def _qset(n, k, bits, seed):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    return workload.quantize_affine(w, 64, bits, torch.bfloat16)


def _deq(qset, bits):
    return workload.dequantize(*qset, 64, bits).float()


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("tp", [2, 4, 8])
def test_shards_dequantise_to_exact_slices(bits, tp):
    full = _qset(256, 1024, bits, seed=tp + bits)
    W = _deq(full, bits)
    for r in range(tp):
        rows = _deq(llama_tp.shard_rows(full, r, tp), bits)
        assert torch.equal(rows, W[r * 256 // tp:(r + 1) * 256 // tp])
        cols = _deq(llama_tp.shard_cols(full, r, tp, 64, bits), bits)
        assert torch.equal(cols, W[:, r * 1024 // tp:(r + 1) * 1024 // tp])


def test_split_rejects_partial_groups():
    full = _qset(64, 192, 8, seed=1)
    with pytest.raises(ValueError):
        llama_tp.shard_cols(full, 0, 2, 64, 8)  # 96 columns per shard is not whole groups of 64
    with pytest.raises(ValueError):
        llama_tp.shard_rows(full, 0, 3)


def test_llama_8b_splits_at_every_tp():
    cfg = llama_tp.LLAMA3_8B
    for tp in (1, 2, 4, 8):
        assert cfg.heads % tp == 0 and cfg.kv_heads % tp == 0
        assert cfg.ffn % (tp * cfg.group) == 0 and cfg.hidden % (tp * cfg.group) == 0
        assert (cfg.ffn // tp) % 128 == 0 and (cfg.kv_heads // tp * cfg.head_dim) % 128 == 0
        assert cfg.vocab % tp == 0


def _worker(rank, world, init_file, q):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    try:
        up, down, head = _qset(512, 256, 8, 3), _qset(256, 512, 8, 4), _qset(96, 256, 8, 5)
        x = torch.randn(6, 256, generator=torch.Generator().manual_seed(7))
        comm = llama_tp.ProcessGroupComm()
        a = x @ _deq(llama_tp.shard_rows(up, rank, world), 8).T
        part = a @ _deq(llama_tp.shard_cols(down, rank, world, 64, 8), 8).T
        y = comm.all_reduce([part])
        logits = comm.all_gather([y @ _deq(llama_tp.shard_rows(head, rank, world), 8).T])
        ref_y = (x @ _deq(up, 8).T) @ _deq(down, 8).T
        ref_logits = ref_y @ _deq(head, 8).T
        ok = (torch.allclose(y, ref_y, rtol=1e-4, atol=1e-6) and logits.shape == ref_logits.shape
              and torch.allclose(logits, ref_logits, rtol=1e-4, atol=1e-6))
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_column_row_pair_over_two_gloo_ranks(tmp_path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    init_file = str(tmp_path / "pg")
    procs = [ctx.Process(target=_worker, args=(r, 2, init_file, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    assert codes == [0, 0], codes
    got = dict(q.get(timeout=5) for _ in range(2))
    assert got == {0: True, 1: True}


def test_forward_flops_llama_8b():
    # projections 2*T*218.1M*32 + causal attention + lm_head
    f = llama_tp.forward_flops(llama_tp.LLAMA3_8B, 8, 2048)
    assert 2.3e14 < f < 2.5e14, f


def test_llama_shards_are_slices_of_one_model():
    """The model-level split on the host: every tp=2 shard of every projection is the
    matching slice of the tp=1 weights (column shards along N, row shards along K),
    heads and lm_head rows divide as the config says."""
    cfg = llama_tp.LlamaConfig(hidden=256, layers=2, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=384)
    full = llama_tp.LlamaTP(cfg, 1, [0], llama_tp.LocalComm(), seed=9, device="cpu")
    split = llama_tp.LlamaTP(cfg, 2, [0, 1], llama_tp.LocalComm(), seed=9, device="cpu")
    assert (split.hq, split.hkv) == (2, 1)
    per = 32 // cfg.bits
    for li in range(cfg.layers):
        f = full.shards[0].layers[li]
        s0, s1 = (sh.layers[li] for sh in split.shards)
        for a, b0, b1 in [(f.qkv[0], s0.qkv[0], s1.qkv[0]), (f.qkv[1], s0.qkv[1], s1.qkv[1]),
                          (f.qkv[2], s0.qkv[2], s1.qkv[2]), (f.gate, s0.gate, s1.gate), (f.up, s0.up, s1.up)]:
            for t, u0, u1 in zip(a, b0, b1):
                assert torch.equal(torch.cat([u0, u1], dim=0), t)
        for a, b0, b1 in [(f.o, s0.o, s1.o), (f.down, s0.down, s1.down)]:
            assert b0[0].shape[1] * per * 2 == a[0].shape[1] * per
            for t, u0, u1 in zip(a, b0, b1):
                assert torch.equal(torch.cat([u0, u1], dim=1), t)
    assert torch.equal(torch.cat([sh.lm_head[0] for sh in split.shards]), full.shards[0].lm_head[0])
    assert split.shards[0].lm_head[0].shape[0] == cfg.vocab // 2
