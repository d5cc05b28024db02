"""Llama tensor-parallel forward over two GPUs with NCCL (skipped on one GPU).

Two ranks each hold one shard on their own GPU and sum the row-parallel
partials with NCCL all-reduce; rank 0 checks the gathered logits against the
same seeded model run unsharded (tp = 1) on its GPU."""
from __future__ import annotations

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _rank(rank, init_file, q):
    import datetime

    import torch.distributed as dist

    from metal_autotune_b200 import lib, workload
    from metal_autotune_b200.targets import llama_tp
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"file://{init_file}", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        cfg = llama_tp.LlamaConfig(hidden=512, layers=2, heads=4, kv_heads=2, head_dim=128, ffn=1024, vocab=1024)
        tok = workload.seeded_tokens((2, 192), 0, cfg.vocab, seed=3, device=f"cuda:{rank}")
        m = llama_tp.LlamaTP(cfg, 2, [rank], llama_tp.ProcessGroupComm(), seed=5, device=f"cuda:{rank}")
        got = m(tok)                      # two micro-batches, all-reduces overlapped with compute
        m.overlap = False
        serial = m(tok)                   # one batch, all-reduces between the blocks
        torch.cuda.synchronize()
        ok = lib.device_status(clear=True) == 0 and tuple(got.shape) == (2, cfg.vocab)
        if rank == 0:
            ref = llama_tp.LlamaTP(cfg, 1, [0], llama_tp.LocalComm(), seed=5, device="cuda:0")(tok)
            for out in (got, serial):
                rel = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
                ok = ok and rel < 1e-2
        dist.barrier()
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_tp2_over_nccl_matches_tp1(cuda, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, str(tmp_path / "pg"), q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        for p in procs:
            p.join(timeout=300)
    finally:
        # a rank still alive (e.g. stuck in a collective) is ended, not left on its GPU
        for p in procs:
            if p.is_alive():
                p.terminate()
                p.join(timeout=10)
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
    assert [p.exitcode for p in procs] == [0, 0]
    assert dict(q.get(timeout=5) for _ in range(2)) == {0: True, 1: True}
