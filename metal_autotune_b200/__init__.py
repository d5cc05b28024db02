"""B200-native (sm_100a) region kernels for the hot path of
shivamg05/metal-autotune: MLX-affine int4/int8 quantized matmul (tcgen05/TMEM
prefill, vector decode), RMSNorm(+residual), RoPE with offset, SwiGLU, causal
GQA attention, GELU-MLP, LayerNorm, the Mamba selective scan and the
output-diff reduction, behind the C ABI of include/mt.h (libmt.so) and the
reference's region contract (autotuner_runtime)."""

__version__ = "0.1.0"
