"""Region wrappers of the Whisper encoder bundle.

In the shape of the reference's generated replay wrappers
(examples/lfm2_5_1_2b_prefill/lfm2_5_1_2b_prefill_artifact/patch/wrappers.py:
38-106): each region is one try_call of a kernel spec; when a region's
predicate covers the call (None), the wrapper runs that region's original
ops from the wrapped module. With MT_STRICT_REGIONS=1 a fallback raises.

Per block: attn_ln | q/k/v projections as one GEMM over the stacked weights
(k's bias zero: the same outputs column for column) | self-attention reading
q, k, v as strided views of that one buffer | out projection + residual |
mlp_ln | fc1 + GELU | fc2 + residual. Around the blocks: conv1 + GELU, conv2 +
GELU, + positional embedding, ln_post.
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


class W_whisper_block(_Counting):
    KERNEL_IDS = ["layer_norm", "qkv_linear", "self_attention", "out_proj_residual", "fc1_gelu", "fc2_residual"]

    def __init__(self, wrapped, specs=None):
        super().__init__(wrapped, specs)
        a = wrapped.attn
        S = a.query.weight.shape[0]
        kb = torch.zeros(S, dtype=a.query.weight.dtype, device=a.query.weight.device)
        object.__setattr__(self, "_w", {
            "qkv_w": torch.cat([a.query.weight, a.key.weight, a.value.weight]).contiguous(),
            "qkv_b": torch.cat([a.query.bias, kb, a.value.bias]).contiguous(),
        })

    def forward(self, x):
        if not (x.dim() == 3 and x.is_cuda and x.dtype in (torch.float16, torch.bfloat16)):
            return self.wrapped(x)
        L = self.wrapped
        a = L.attn
        cfg = a.cfg
        B, T, S = x.shape
        W = self._w
        r = self._call("layer_norm", [x, L.attn_ln.weight, L.attn_ln.bias])
        h = r[0] if r is not None else L.attn_ln(x)
        r = self._call("qkv_linear", [h, W["qkv_w"], W["qkv_b"]])
        if r is not None:
            qkv = r[0]
            heads = lambda j: qkv[:, :, j * S:(j + 1) * S].view(B, T, cfg.n_head, cfg.head_dim)
            r = self._call("self_attention", [heads(0), heads(1), heads(2)])
            o = r[0] if r is not None else a.attend(qkv[:, :, :S], qkv[:, :, S:2 * S], qkv[:, :, 2 * S:])
        else:
            o = a.attend(a.query(h), a.key(h), a.value(h))
        r = self._call("out_proj_residual", [o, a.out.weight, a.out.bias, x])
        x = r[0] if r is not None else (x.float() + a.out(o).float()).to(x.dtype)
        r = self._call("layer_norm", [x, L.mlp_ln.weight, L.mlp_ln.bias])
        h = r[0] if r is not None else L.mlp_ln(x)
        r = self._call("fc1_gelu", [h, L.mlp1.weight, L.mlp1.bias])
        if r is None:
            from metal_autotune_b200.targets.whisper import gelu
            r = [gelu(L.mlp1(h))]
        r2 = self._call("fc2_residual", [r[0], L.mlp2.weight, L.mlp2.bias, x])
        return r2[0] if r2 is not None else (x.float() + L.mlp2(r[0]).float()).to(x.dtype)


class W_whisper_encoder(_Counting):
    KERNEL_IDS = ["conv1_gelu", "conv2_gelu", "pos_add", "layer_norm"]

    def forward(self, mel):
        E = self.wrapped
        r = self._call("conv1_gelu", [mel, E.conv1.weight, E.conv1.bias])
        if r is None:
            from metal_autotune_b200.targets.whisper import gelu
            r = [gelu(E.conv1(mel))]
        x = r[0]
        r = self._call("conv2_gelu", [x, E.conv2.weight, E.conv2.bias])
        if r is None:
            from metal_autotune_b200.targets.whisper import gelu
            r = [gelu(E.conv2(x))]
        x = r[0]
        r = self._call("pos_add", [x, E.positional_embedding])
        x = r[0] if r is not None else (x.float() + E.positional_embedding.float()).to(x.dtype)
        for blk in E.blocks:
            x = blk(x)
        r = self._call("layer_norm", [x, E.ln_post.weight, E.ln_post.bias])
        return r[0] if r is not None else E.ln_post(x)
