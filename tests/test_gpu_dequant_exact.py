"""Bit-exact dequantisation on the prefill (tensor-core) qmm path.

The prefill kernel dequantises each weight tile to the activation dtype with
MLX's rounding, round(round(scale * q) + bias), before the tensor-core MMA.
Multiplying by one-hot rows isolates that step: with x = I (M = K rows, a
single 1.0 per row) every output is one dequantised weight times 1.0 plus
exact zeros, accumulated in fp32 and rounded back to the weight's own dtype,
so y[i, n] must equal dequant(w)[n, i] bit for bit (up to the sign of zero:
-0.0 + 0.0 sums to +0.0). M = K >= 512 keeps every call on the tcgen05 path
(the vector path serves M <= 8)."""
import numpy as np
import pytest
import torch

from metal_autotune_b200 import lib

from test_gpu_kernels import quantized, t

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("N,K,group", [(256, 512, 64), (200, 1024, 64), (384, 512, 32), (256, 1024, 128)])
def test_prefill_qmm_dequant_bit_exact(cuda, oracle, dtype, bits, N, K, group):
    tdt = torch.bfloat16 if dtype == "bfloat16" else torch.float16
    (wq, s, b), (wq_t, s_t, b_t) = quantized(oracle, N, K, group, bits, dtype, seed=N + K + bits)
    eye = torch.eye(K, device="cuda", dtype=tdt)
    y = lib.quantized_matmul(eye, wq_t, s_t, b_t, group_size=group, bits=bits)
    torch.cuda.synchronize()
    got = y.float().cpu().numpy()                       # [K, N]: row i is column i of W
    want = oracle.dequantize(wq, s, b, group, bits, dtype).T
    want = want + np.float32(0.0)                       # -0.0 -> +0.0, as the fp32 sum gives
    assert got.dtype == want.dtype == np.float32
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"{int((got != want).sum())} of {got.size} dequantised weights differ"
