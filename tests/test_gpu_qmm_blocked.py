"""Parity of the blocked tensor-core qmm path (large M x N split into L2-sized
launches) with the CPU oracle.

MT_QMM_L2_BLOCK_BYTES is set small here so that moderate sizes split into
several token-row and weight-row blocks: ragged last blocks, the SwiGLU pair
split by weight rows, the q/k/v triple split by token rows only, the residual
carried at the full row pitch. Tolerances as in test_gpu_kernels.py."""
import numpy as np
import pytest
import torch

from metal_autotune_b200 import lib

from test_gpu_kernels import close_bf16, n, quantized, t

pytestmark = pytest.mark.gpu

rng = np.random.default_rng(99)
BUDGET = str(256 * 1024)  # 128 token rows x 1024 K per block; 128-384 weight rows


@pytest.fixture
def small_blocks(monkeypatch):
    monkeypatch.setenv("MT_QMM_L2_BLOCK_BYTES", BUDGET)


@pytest.mark.parametrize("M,N,K,bits", [(600, 640, 1024, 8), (257, 520, 512, 4), (384, 256, 2048, 8)])
def test_blocked_plain_and_residual(cuda, oracle, small_blocks, M, N, K, bits):
    x = oracle.round_to(rng.standard_normal((M, K)).astype(np.float32), "bfloat16")
    r = oracle.round_to(rng.standard_normal((M, N)).astype(np.float32), "bfloat16")
    (wq, s, b), (wq_t, s_t, b_t) = quantized(oracle, N, K, 64, bits)
    ref = oracle.quantized_matmul(x, wq, s, b, 64, bits)
    y = lib.quantized_matmul(t(x), wq_t, s_t, b_t, bits=bits)
    torch.cuda.synchronize()
    close_bf16(n(y), ref, ulps=1)
    yr = lib.quantized_matmul(t(x), wq_t, s_t, b_t, bits=bits, residual=t(r))
    close_bf16(n(yr), oracle.add(ref, r), ulps=2)
    assert lib.device_status(clear=True) == 0


def test_blocked_swiglu(cuda, oracle, small_blocks):
    M, N, K = 300, 896, 1024
    x = oracle.round_to(rng.standard_normal((M, K)).astype(np.float32), "bfloat16")
    (wg, sg, bg), gt = quantized(oracle, N, K, 64, 8, seed=1)
    (wu, su, bu), ut = quantized(oracle, N, K, 64, 8, seed=2)
    y = lib.quantized_matmul_swiglu(t(x), *gt, *ut, bits=8)
    g = oracle.quantized_matmul(x, wg, sg, bg, 64, 8)
    u = oracle.quantized_matmul(x, wu, su, bu, 64, 8)
    close_bf16(n(y), oracle.swiglu(g, u), ulps=3, abs_frac=2 ** -8)


def test_blocked_multi(cuda, oracle, small_blocks):
    M, K = 400, 1024
    x = oracle.round_to(rng.standard_normal((M, K)).astype(np.float32), "bfloat16")
    sets = [quantized(oracle, Nn, K, 64, 8, seed=10 + i) for i, Nn in enumerate((512, 128, 128))]
    ys = lib.quantized_matmul_multi(t(x), [g for _, g in sets], bits=8)
    for ((wq, s, b), _), y in zip(sets, ys):
        close_bf16(n(y), oracle.quantized_matmul(x, wq, s, b, 64, 8), ulps=1)


def test_blocked_equals_one_launch_within_tolerance(cuda, oracle, monkeypatch):
    """The same product with and without blocking: both within tolerance of each other."""
    M, N, K = 512, 768, 1024
    x = t(oracle.round_to(rng.standard_normal((M, K)).astype(np.float32), "bfloat16"))
    _, (wq_t, s_t, b_t) = quantized(oracle, N, K, 64, 8)
    one = lib.quantized_matmul(x, wq_t, s_t, b_t, bits=8)
    monkeypatch.setenv("MT_QMM_L2_BLOCK_BYTES", BUDGET)
    blocked = lib.quantized_matmul(x, wq_t, s_t, b_t, bits=8)
    close_bf16(n(blocked), n(one), ulps=1)


@pytest.mark.parametrize("empty", [(0,), (0, 2), (0, 1)])
def test_blocked_multi_with_empty_leading_sets(cuda, oracle, small_blocks, empty):
    """mt_quantized_matmul_multi with set 0 (and possibly another) left empty:
    the blocked path splits by the first set that has rows."""
    M, K, N = 300, 1024, 640
    x = oracle.round_to(rng.standard_normal((M, K)).astype(np.float32), "bfloat16")
    xt = t(x)
    live = [i for i in range(3) if i not in empty]
    sets = {i: quantized(oracle, N, K, 64, 8, seed=20 + i) for i in live}
    ys = {i: torch.empty(M, N, dtype=torch.bfloat16, device="cuda") for i in live}
    args = []
    for i in range(3):
        if i in sets:
            w, s, b = sets[i][1]
            args += [lib._ptr(w), lib._ptr(s), lib._ptr(b), lib._ptr(ys[i]), N]
        else:
            args += [None, None, None, None, 0]
    ws = lib.Workspace.get(lib.qmm_workspace_bytes(M, N * len(live), K, 8, 0))
    lib.call("mt_quantized_matmul_multi", lib._ptr(xt), *args, M, K, 64, 8, lib.MT_BF16, ws.ptr, ws.nbytes,
             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    for i in live:
        wq, s, b = sets[i][0]
        close_bf16(n(ys[i]), oracle.quantized_matmul(x, wq, s, b, 64, 8), ulps=1)
