"""Region wrappers of the Mamba bundle.

In the shape of the reference's generated replay wrappers
(examples/lfm2_5_1_2b_prefill/lfm2_5_1_2b_prefill_artifact/patch/wrappers.py:
38-106): each region is one try_call of a kernel spec, the wrapped module's
original ops when a region's predicate covers the call (None). With
MT_STRICT_REGIONS=1 a fallback raises.

Per layer: rms_norm | in_proj as two GEMMs (the x and z halves of its
weight rows, so each half is a contiguous operand) | depthwise causal conv +
SiLU | x_proj as three GEMMs (delta, B, C rows) | dt_proj + bias | selective
scan with the SiLU(z) gate | out_proj + residual. Around the layers: the
embedding gather, norm_f on the last position, the tied lm_head and the
greedy pick.
"""
import os

import torch

from metal_autotune_b200.autotuner_runtime import kernels as _kernels
from metal_autotune_b200.autotuner_runtime.swap import ReplayWrapper


def _strict() -> bool:
    return os.environ.get("MT_STRICT_REGIONS", "0") == "1"


class _Counting(ReplayWrapper):
    def __init__(self, wrapped, specs=None):
        super().__init__(wrapped, specs)
        object.__setattr__(self, "fallbacks", 0)

    def _call(self, kid, inputs):
        out = _kernels.try_call(self._specs[kid], inputs)
        if out is None:
            if _strict():
                raise RuntimeError(f"region {kid} fell back to the original ops")
            object.__setattr__(self, "fallbacks", self.fallbacks + 1)
        return out


class W_mamba_layer(_Counting):
    KERNEL_IDS = ["rms_norm", "linear", "linear_bias", "causal_conv1d_silu", "selective_scan", "out_proj_residual"]

    def __init__(self, wrapped, specs=None):
        super().__init__(wrapped, specs)
        m = wrapped.mixer
        cfg = m.cfg
        E, Rk, S = cfg.d_inner, cfg.dt_rank, cfg.d_state
        object.__setattr__(self, "_w", {
            "in_x": m.in_proj[:E].contiguous(), "in_z": m.in_proj[E:].contiguous(),
            "xp_delta": m.x_proj[:Rk].contiguous(), "xp_B": m.x_proj[Rk:Rk + S].contiguous(),
            "xp_C": m.x_proj[Rk + S:].contiguous(),
            "A": (-torch.exp(m.A_log.float())).contiguous(), "D": m.D.float().contiguous(),
        })

    def forward(self, x):
        if not (x.dim() == 2 and x.is_cuda and x.dtype in (torch.float16, torch.bfloat16)):
            return self.wrapped(x)
        L = self.wrapped
        m = L.mixer
        W = self._w
        r = self._call("rms_norm", [x, L.norm.weight])
        h = r[0] if r is not None else L.norm(x)
        outs = []
        for key in ("in_x", "in_z"):
            r = self._call("linear", [h, W[key]])
            outs.append(r[0] if r is not None else (h.float() @ W[key].float().t()).to(h.dtype))
        xs, z = outs
        r = self._call("causal_conv1d_silu", [xs, m.conv_w, m.conv_b])
        xc = r[0] if r is not None else m.conv(xs)
        parts = []
        for key in ("xp_delta", "xp_B", "xp_C"):
            r = self._call("linear", [xc, W[key]])
            parts.append(r[0] if r is not None else (xc.float() @ W[key].float().t()).to(xc.dtype))
        delta, B, C = parts
        r = self._call("linear_bias", [delta, m.dt_proj, m.dt_bias])
        dt = r[0] if r is not None else ((delta.float() @ m.dt_proj.float().t()) + m.dt_bias.float()).to(xc.dtype)
        r = self._call("selective_scan", [xc, dt, W["A"], B, C, W["D"], z])
        y = r[0] if r is not None else m.scan(xc, dt, B, C, z)
        r = self._call("out_proj_residual", [y, m.out_proj, x])
        return r[0] if r is not None else (x.float() + (y.float() @ m.out_proj.float().t()).to(x.dtype).float()).to(x.dtype)


class W_mamba_model(_Counting):
    KERNEL_IDS = ["embedding", "rms_norm", "linear", "logits_pick"]

    def forward(self, tokens):
        M = self.wrapped
        r = self._call("embedding", [tokens, M.embedding])
        x = r[0] if r is not None else M.embedding[tokens.long()]
        for layer in M.layers:
            x = layer(x)
        last = x[-1:]
        r = self._call("rms_norm", [last, M.norm_f.weight])
        h = r[0] if r is not None else M.norm_f(last)
        r = self._call("linear", [h, M.embedding])
        logits = r[0] if r is not None else (h.float() @ M.embedding.float().t()).to(h.dtype)
        object.__setattr__(self, "last_logits", logits)
        r = self._call("logits_pick", [logits])
        if r is None:
            return torch.argmax(logits.float(), dim=-1).to(torch.int32), logits
        return r[0], logits
