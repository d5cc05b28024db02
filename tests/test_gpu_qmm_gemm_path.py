"""Parity of the many-rows form of the quantized matmul family: from 1024 rows
of x up, the weights are dequantised once into the workspace and multiplied
on the tcgen05 GEMM. Checked against the fused tensor-core kernel on the same
inputs (MT_QMM_GEMM_MIN_ROWS pushes the threshold out of reach for the
reference run) and against an fp32 torch product of the MLX-dequantised
weights, within one element-type ulp of the value plus 2^-9 of the largest
magnitude; the dequantisation itself bit for bit through one-hot rows."""
from __future__ import annotations

import pytest
import torch

from metal_autotune_b200 import lib, workload

pytestmark = pytest.mark.gpu


def _close(got, want, dtype):
    ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10
    g, w = got.float(), want.float()
    tol = ulp * w.abs() + 2.0 ** -9 * w.abs().max()
    bad = (g - w).abs() > tol
    assert not bad.any(), f"{int(bad.sum())} of {w.numel()} elements off (max diff {(g - w).abs().max():.3g})"


def _fused_and_gemm(fn, monkeypatch):
    monkeypatch.setenv("MT_QMM_GEMM_MIN_ROWS", str(1 << 40))
    fused = [t.clone() for t in fn()]
    monkeypatch.delenv("MT_QMM_GEMM_MIN_ROWS")
    gemm = [t.clone() for t in fn()]
    return fused, gemm


def _weights(N, K, bits, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return workload.random_quantized(N, K, bits=bits, dtype=dtype, generator=g)


def _x(M, K, dtype, seed):
    return torch.randn(M, K, generator=torch.Generator().manual_seed(seed)).to(dtype).cuda()


@pytest.mark.parametrize("M,N,K,bits,dtype", [(1024, 384, 512, 4, torch.bfloat16), (1500, 200, 1024, 8, torch.bfloat16),
                                             (1024, 256, 512, 4, torch.float16)])
def test_plain_and_residual(cuda, monkeypatch, M, N, K, bits, dtype):
    w = _weights(N, K, bits, dtype, 1)
    x, r = _x(M, K, dtype, 2), _x(M, N, dtype, 3)
    ref = torch.matmul(x.float(), workload.dequantize(*w, 64, bits).float().t())
    fused, gemm = _fused_and_gemm(lambda: [lib.quantized_matmul(x, *w, bits=bits),
                                           lib.quantized_matmul(x, *w, bits=bits, residual=r)], monkeypatch)
    _close(gemm[0], fused[0], dtype)
    _close(gemm[0], ref.to(dtype), dtype)
    _close(gemm[1], fused[1], dtype)
    _close(gemm[1], (ref.to(dtype).float() + r.float()).to(dtype), dtype)


def test_three_projections_and_swiglu(cuda, monkeypatch):
    """Several sets share one dequantisation buffer in turn; the SwiGLU pair
    is one GEMM over gate and up rows interleaved in 128-row blocks, SwiGLU in
    its epilogue (320 outputs: a partial last block)."""
    M, K, bits, dtype = 1152, 512, 4, torch.bfloat16
    sets = [_weights(n, K, bits, dtype, 10 + i) for i, n in enumerate((256, 128, 64))]
    x = _x(M, K, dtype, 4)
    fused, gemm = _fused_and_gemm(lambda: lib.quantized_matmul_multi(x, sets, bits=bits), monkeypatch)
    for f, g in zip(fused, gemm):
        _close(g, f, dtype)
    wg, wu = _weights(320, K, bits, dtype, 20), _weights(320, K, bits, dtype, 21)
    fused, gemm = _fused_and_gemm(lambda: [lib.quantized_matmul_swiglu(x, *wg, *wu, bits=bits)], monkeypatch)
    _close(gemm[0], fused[0], dtype)


@pytest.mark.parametrize("bits,dtype", [(4, torch.bfloat16), (8, torch.bfloat16), (4, torch.float16),
                                        (8, torch.float16)])
def test_dequantisation_is_exact_through_one_hot_rows(cuda, bits, dtype):
    """x = I (1024 one-hot rows): every output is one product of 1 with a
    dequantised weight, so y = dequant(W)^T bit for bit."""
    K = N = 1024
    w = _weights(N, K, bits, dtype, 5)
    x = torch.eye(K, dtype=dtype, device="cuda")
    y = lib.quantized_matmul(x, *w, bits=bits)
    assert torch.equal(y, workload.dequantize(*w, 64, bits).t().contiguous())


def test_workspace_query_grows_only_from_the_threshold():
    small = lib.qmm_workspace_bytes(1023, 4096, 4096, 4, 0)
    large = lib.qmm_workspace_bytes(1024, 4096, 4096, 4, 0)
    assert large >= small + 4096 * 4096 * 2
    dual = lib.qmm_workspace_bytes(2048, 2 * 1000, 512, 4, 1)
    assert dual >= 256 * 8 * 512 * 2  # 1000 outputs: 8 blocks of 128 gate + 128 up rows


def test_the_path_launches_dequantisation_and_gemm(cuda):
    """One set: a dequantisation pass and a GEMM; SwiGLU: a pass per set and
    one GEMM (mt_kernel_launches counts every kernel libmt launches)."""
    M, K, bits, dtype = 1024, 512, 4, torch.bfloat16
    x = _x(M, K, dtype, 6)
    w, wg, wu = (_weights(256, K, bits, dtype, 30 + i) for i in range(3))
    n0 = lib.kernel_launches()
    lib.quantized_matmul(x, *w, bits=bits)
    n1 = lib.kernel_launches()
    lib.quantized_matmul_swiglu(x, *wg, *wu, bits=bits)
    n2 = lib.kernel_launches()
    torch.cuda.synchronize()
    assert (n1 - n0, n2 - n1) == (2, 3)
