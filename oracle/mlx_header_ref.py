"""TEST INFRASTRUCTURE — a second oracle path for the quantised matmul: the
MLX-derived arithmetic the reference itself holds.

The reference stores no golden outputs, but one of its shipped artifacts
carries MLX's own dequantisation and decode dot-product arithmetic as Metal
helpers: the header of
examples/lfm2_5_1_2b_prefill/lfm2_5_1_2b_prefill_artifact/kernels/
r1f9367e50750eb01_unroll_hoist.launch.json ("header": `mlx_deq8`,
`qmv_qdot16`; the M < 6 branch of its "source" shows how qmv_qdot16 is
driven). This module restates that arithmetic in numpy, for 4-bit group-64
weights with bf16 scales, biases and activations:

  dequant (mlx_deq8): per packed byte, the low nibble q_lo and the high nibble
    kept in place (16 q_hi); w_lo = bf16(bf16(s * q_lo) + b) and
    w_hi = bf16(bf16((s / 16) * (16 q_hi)) + b): every operation a bf16 op
    (computed in fp32, rounded to bf16).
  qmv (qmv_qdot16): x is read in chunks of 16 values. Per chunk,
    sum = sum over its four quads of fp32(bf16(bf16(bf16(h0 + h1) + h2) + h3)),
    xt = (h0, h1 / 16, h2 / 256, h3 / 4096) per quad, and each packed
    half-word's four nibbles are used in place (masks 0xF, 0xF0, 0xF00,
    0xF000), so xt * masked = x * q exactly; accum = sum over the chunk of
    those products (fp32), chunk value = s * accum + sum * b. Lane l of a
    32-lane group takes chunks l, l + 32, l + 64, ... in order; the lanes'
    totals are then summed (simd_sum; restated as a pairwise tree) and
    rounded to bf16.

Used by the tests only, as an independent check of oracle/mt_oracle.c and of
the GPU kernels; the fp32 summation orders differ, so qmv agrees within a
tolerance and the dequantised weights bit for bit.
"""
from __future__ import annotations

import numpy as np

from .ref import round_to

F32 = np.float32


def _bf(a) -> np.ndarray:
    return round_to(np.asarray(a, F32), "bfloat16")


def deq8(wq: np.ndarray, scales: np.ndarray, biases: np.ndarray, group: int = 64) -> np.ndarray:
    """Dequantised [N, K] (4-bit, bf16 scale/bias) by the mlx_deq8 arithmetic."""
    wq = np.asarray(wq, np.uint32)
    N, words = wq.shape
    K = words * 8
    bytes_ = ((wq[:, :, None] >> (np.arange(4, dtype=np.uint32) * 8)) & 0xFF).reshape(N, K // 2)
    lo = (bytes_ & 0x0F).astype(F32)
    hi16 = (bytes_ & 0xF0).astype(F32)          # 16 * q_hi, exact in bf16
    s = np.repeat(_bf(scales), group // 2, axis=1)  # one scale per packed byte (two values)
    b = np.repeat(_bf(biases), group // 2, axis=1)
    sc1 = _bf(s / F32(16.0))
    w = np.empty((N, K), F32)
    w[:, 0::2] = _bf(_bf(s * lo) + b)
    w[:, 1::2] = _bf(_bf(sc1 * hi16) + b)
    return w


def qmv_qdot16(x: np.ndarray, wq: np.ndarray, scales: np.ndarray, biases: np.ndarray, group: int = 64,
               bf16_quad_sums: bool = True) -> np.ndarray:
    """y [M, N] for bf16 x [M, K] by the qmv_qdot16 arithmetic (4-bit, g64).

    bf16_quad_sums=False sums each quad of x in fp32 instead: the same
    factored form without the bf16 rounding of the quad sums, which is the
    one step where MLX's qmv knowingly rounds more than the factored fp32
    form (the oracle's qmv and the GPU decode kernels sum x in fp32)."""
    assert group == 64
    x = _bf(np.asarray(x, F32))
    M, K = x.shape
    wq = np.asarray(wq, np.uint32)
    N = wq.shape[0]
    assert K % 512 == 0, "the restated lane schedule covers K in steps of 32 lanes x 16 values"
    chunks = K // 16
    s = _bf(scales)[:, np.arange(chunks) * 16 // 64]        # [N, chunks]
    b = _bf(biases)[:, np.arange(chunks) * 16 // 64]
    # nibble values in place: q * 16^(position in its quad)
    nib = ((wq[:, :, None] >> (np.arange(8, dtype=np.uint32) * 4)) & 0xF).reshape(N, K)
    place = np.tile(np.array([1, 16, 256, 4096], F32), K // 4)
    masked = nib.astype(F32) * place                          # exact
    out = np.empty((M, N), F32)
    for m in range(M):
        h = x[m].reshape(chunks, 4, 4)                        # chunk, quad, value
        if bf16_quad_sums:
            hs = _bf(_bf(_bf(h[:, :, 0] + h[:, :, 1]) + h[:, :, 2]) + h[:, :, 3])
        else:
            hs = ((h[:, :, 0] + h[:, :, 1]).astype(F32) + h[:, :, 2]).astype(F32) + h[:, :, 3]
        sums = np.zeros(chunks, F32)
        for qd in range(4):
            sums = (sums + hs[:, qd]).astype(F32)
        xt = (x[m].reshape(K // 4, 4) / np.array([1, 16, 256, 4096], F32)).reshape(K).astype(F32)
        prod = (masked * xt[None, :]).reshape(N, chunks, 4, 4)  # exact products
        acc = np.zeros((N, chunks), F32)
        for qd in range(4):
            quad = prod[:, :, qd, :]
            t = ((quad[..., 0] + quad[..., 1]).astype(F32) + quad[..., 2]).astype(F32) + quad[..., 3]
            acc = (acc + t.astype(F32)).astype(F32)
        val = (s * acc).astype(F32) + (sums[None, :] * b).astype(F32)
        val = val.astype(F32)
        lanes = np.zeros((N, 32), F32)
        for j in range(chunks // 32):
            lanes = (lanes + val[:, j * 32:(j + 1) * 32]).astype(F32)
        width = 32
        while width > 1:                                      # pairwise tree over the lanes
            width //= 2
            lanes = (lanes[:, :width] + lanes[:, width:2 * width]).astype(F32)
        out[m] = lanes[:, 0]
    return _bf(out)


def quad_sum_sigma(x: np.ndarray, biases: np.ndarray, group: int = 64) -> np.ndarray:
    """[M, N] standard deviation of the difference the bf16 quad sums make:
    each of the three bf16 additions of a quad rounds with an error uniform
    within half an ulp of its result (variance ulp^2 / 12), and the quad's
    error enters the output multiplied by its group's bias."""
    x = _bf(np.asarray(x, F32))
    M, K = x.shape
    q = x.reshape(M, K // 4, 4).astype(np.float64)
    partial = np.stack([q[..., 0] + q[..., 1], q[..., 0] + q[..., 1] + q[..., 2], q.sum(-1)], axis=-1)
    mag = np.maximum(np.abs(partial), 2.0 ** -133)
    ulp = 2.0 ** (np.floor(np.log2(mag)) - 7)                # bf16 ulp of each partial sum
    var_quad = (ulp ** 2 / 12).sum(-1)                       # [M, K/4]
    var_group = var_quad.reshape(M, K // group, group // 4).sum(-1)   # [M, G]
    b2 = np.asarray(biases, np.float64) ** 2                 # [N, G]
    return np.sqrt(var_group @ b2.T)
