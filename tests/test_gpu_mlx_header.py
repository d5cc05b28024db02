"""The GPU quantised matmul against the second oracle path: the MLX-derived
dequantisation and decode arithmetic the reference holds in its LFM2
artifact header (mlx_deq8, qmv_qdot16; oracle/mlx_header_ref.py).

- prefill (tcgen05 path): x = I isolates the dequantisation, which must equal
  mlx_deq8 bit for bit;
- decode (M <= 8, the streamed and plain vector kernels): the factored form
  with fp32 quad sums within one bf16 ulp plus 2^-9 of the row scale, and
  MLX's bf16 quad sums within that plus 6 standard deviations of their
  rounding noise (quad_sum_sigma)."""
import numpy as np
import pytest
import torch

from metal_autotune_b200 import lib

from test_gpu_kernels import quantized, t

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("N,K", [(256, 512), (192, 2560)])
def test_prefill_dequant_equals_mlx_deq8(cuda, oracle, N, K):
    from oracle import mlx_header_ref as H
    (wq, s, b), (wq_t, s_t, b_t) = quantized(oracle, N, K, 64, 4, seed=N * 7 + K)
    y = lib.quantized_matmul(torch.eye(K, device="cuda", dtype=torch.bfloat16), wq_t, s_t, b_t)
    got = y.float().cpu().numpy().T
    want = H.deq8(wq, s, b, 64) + np.float32(0.0)  # -0.0 -> +0.0 as the fp32 accumulation gives
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("M,N,K", [(1, 2560, 2560), (1, 1024, 9728), (2, 512, 4096), (4, 640, 2560),
                                   (8, 256, 2560)])
def test_decode_qmv_against_mlx_qdot16(cuda, oracle, M, N, K):
    from oracle import mlx_header_ref as H
    rng = np.random.default_rng(M * 1000 + K)
    x = oracle.round_to(rng.standard_normal((M, K)).astype(np.float32), "bfloat16")
    (wq, s, b), (wq_t, s_t, b_t) = quantized(oracle, N, K, 64, 4, seed=K + N)
    got = lib.quantized_matmul(t(x), wq_t, s_t, b_t).float().cpu().numpy()
    same_form = H.qmv_qdot16(x, wq, s, b, 64, bf16_quad_sums=False)
    tol = 2 ** -7 * np.abs(same_form) + 2 ** -9 * np.abs(same_form).max()
    assert (np.abs(got - same_form) <= tol).all(), np.abs(got - same_form).max()
    mlx = H.qmv_qdot16(x, wq, s, b, 64)
    tol = 2 ** -7 * np.abs(mlx) + 2 ** -9 * np.abs(mlx).max() + 6 * H.quad_sum_sigma(x, b, 64)
    assert (np.abs(got - mlx) <= tol).all(), np.abs(got - mlx).max()
