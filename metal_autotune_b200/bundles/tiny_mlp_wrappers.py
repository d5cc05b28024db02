"""Region wrappers of the tiny GELU-MLP bundle: the first linear with its
bias and GELU as one region, the second linear with its bias as another
(fp32, sequential-k sums), each falling back to the wrapped module's own ops
when its predicate covers the call."""
import math
import os

import torch

from metal_autotune_b200.autotuner_runtime import kernels as _kernels
from metal_autotune_b200.autotuner_runtime.swap import ReplayWrapper


class W_tiny_mlp(ReplayWrapper):
    KERNEL_IDS = ["linear_gelu_f32", "linear_f32"]

    def __init__(self, wrapped, specs=None):
        super().__init__(wrapped, specs)
        object.__setattr__(self, "fallbacks", 0)

    def _call(self, kid, inputs):
        out = _kernels.try_call(self._specs[kid], inputs)
        if out is None:
            if os.environ.get("MT_STRICT_REGIONS", "0") == "1":
                raise RuntimeError(f"region {kid} fell back to the original ops")
            object.__setattr__(self, "fallbacks", self.fallbacks + 1)
        return out

    def forward(self, x):
        m = self.wrapped
        r = self._call("linear_gelu_f32", [x, m.l1.weight, m.l1.bias])
        if r is None:
            h = m.l1(x)
            r = [h * (1 + torch.erf(h / math.sqrt(2))) / 2]
        r2 = self._call("linear_f32", [r[0], m.l2.weight, m.l2.bias])
        return r2[0] if r2 is not None else m.l2(r[0])
