"""Region contract of shivamg05/metal-autotune (its autotuner_runtime
package) re-hosted on PyTorch + libmt.so: KernelSpec and the call site
(kernels), launch grammar, stage dataflow, module swap / apply, captured
kernel definitions, the output contract (numeric, exact) on the GPU diff
reduction, paired statistics and the CUDA-event timing harness."""
from . import grammar, kernels, stages, swap  # noqa: F401
