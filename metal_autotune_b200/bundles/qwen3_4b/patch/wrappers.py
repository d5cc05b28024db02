"""Region wrappers of the Qwen3 bundle.

Hand-written in the shape of the reference's generated replay wrappers
(examples/lfm2_5_1_2b_prefill/lfm2_5_1_2b_prefill_artifact/patch/wrappers.py:
38-106): each region is one try_call of a kernel spec; when its fallback
predicate covers the call (None), the wrapper runs that region's original
ops from the wrapped module. Fallbacks are counted on the wrapper; with
MT_STRICT_REGIONS=1 a fallback raises instead, so a benchmark can prove every
region ran on its kernel.

At decode (at most 4 tokens) the RMSNorm and the matmul after it run as one
fused cut (rms_norm_qkv_qmm, rms_norm_gate_up_swiglu, rms_norm_lm_head), and
the attention prologue and attention as one (qk_norm_rope_sdpa_decode); their
predicates send prefill shapes to the two-region path, which is not a
fallback.
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

    def _call(self, kid, inputs, scalars=None):
        out = _kernels.try_call(self._specs[kid], inputs, scalars=scalars)
        if out is None:
            if _strict():
                raise RuntimeError(f"region {kid} fell back to the original ops")
            object.__setattr__(self, "fallbacks", self.fallbacks + 1)
        return out

    def _fused(self, kid, inputs):
        """The fused decode cut, or None when its predicate sends these shapes
        to the unfused regions."""
        return _kernels.try_call(self._specs[kid], inputs)


class W_qwen3_layer(_Counting):
    """One decoder layer: rms_norm | qkv | q/k norm + rope + cache | sdpa |
    o_proj + residual | rms_norm | gate/up + swiglu | down + residual."""

    KERNEL_IDS = ["rms_norm", "qkv_qmm", "qk_norm_rope_cache", "sdpa_causal_gqa", "o_proj_residual",
                  "gate_up_swiglu", "down_proj_residual", "rms_norm_qkv_qmm", "rms_norm_gate_up_swiglu",
                  "qk_norm_rope_sdpa_decode"]

    def __init__(self, wrapped, specs=None):
        super().__init__(wrapped, specs)
        a, m = wrapped.self_attn, wrapped.mlp
        object.__setattr__(self, "_w", {
            "in_norm": wrapped.input_layernorm.weight,
            "post_norm": wrapped.post_attention_layernorm.weight,
            "qkv": [a.q_proj.weight, a.q_proj.scales, a.q_proj.biases, a.k_proj.weight, a.k_proj.scales,
                    a.k_proj.biases, a.v_proj.weight, a.v_proj.scales, a.v_proj.biases],
            "qk_norm": [a.q_norm.weight, a.k_norm.weight],
            "o": [a.o_proj.weight, a.o_proj.scales, a.o_proj.biases],
            "gate_up": [m.gate_proj.weight, m.gate_proj.scales, m.gate_proj.biases, m.up_proj.weight,
                        m.up_proj.scales, m.up_proj.biases],
            "down": [m.down_proj.weight, m.down_proj.scales, m.down_proj.biases],
        })

    def forward(self, h, cache):
        if not (h.dim() == 2 and h.is_cuda and h.dtype in (torch.bfloat16, torch.float16)):
            return self.wrapped(h, cache)
        W, L = self._w, self.wrapped
        a, m = L.self_attn, L.mlp
        T = h.shape[0]
        off = cache.offset
        r = self._fused("rms_norm_qkv_qmm", [h, W["in_norm"], *W["qkv"]])
        if r is None:
            r = self._call("rms_norm", [h, W["in_norm"]])
            xn = r[0] if r is not None else L.input_layernorm(h)
            r = self._call("qkv_qmm", [xn, *W["qkv"]])
            if r is None:
                r = a.qkv(xn)
        q, k, v = r
        r = _kernels.try_call(self._specs["qk_norm_rope_sdpa_decode"], [q, k, v, *W["qk_norm"], cache.k, cache.v],
                              scalars={"offset": off})
        if r is None:
            r = self._call("qk_norm_rope_cache", [q, k, v, *W["qk_norm"], cache.k, cache.v], {"offset": off})
            qh = r[0] if r is not None else a.prologue(q, k, v, cache)
            r = self._call("sdpa_causal_gqa", [qh, cache.k, cache.v], {"offset": off, "kv_len": off + T})
            if r is None:
                r = [a.attend(qh, cache, off + T)]
        o = r[0]
        r = self._call("o_proj_residual", [o, *W["o"], h])
        h2 = r[0] if r is not None else h + a.o_proj(o)
        r = self._fused("rms_norm_gate_up_swiglu", [h2, W["post_norm"], *W["gate_up"]])
        if r is None:
            r = self._call("rms_norm", [h2, W["post_norm"]])
            xn2 = r[0] if r is not None else L.post_attention_layernorm(h2)
            r = self._call("gate_up_swiglu", [xn2, *W["gate_up"]])
            if r is None:
                r = [m.gate_up(xn2)]
        act = r[0]
        r = self._call("down_proj_residual", [act, *W["down"], h2])
        return r[0] if r is not None else h2 + m.down_proj(act)


class W_qwen3_root(_Counting):
    """Embedding gather, the (wrapped) layers, final norm on the last row,
    tied lm_head and the greedy pick (mlx-lm generate_step)."""

    KERNEL_IDS = ["quantized_embedding", "rms_norm", "lm_head", "logits_pick", "rms_norm_lm_head"]

    def forward(self, tokens, cache):
        M = self.wrapped
        E = M.embed_tokens
        T = tokens.shape[0]
        r = self._call("quantized_embedding", [tokens, E.weight, E.scales, E.biases])
        h = r[0] if r is not None else E(tokens)
        for layer, c in zip(M.layers, cache.layers):
            h = layer(h, c)
        for c in cache.layers:
            c.offset += T
        last = h[-1:]
        r = self._fused("rms_norm_lm_head", [last, M.norm.weight, E.weight, E.scales, E.biases])
        if r is None:
            r = self._call("rms_norm", [last, M.norm.weight])
            xn = r[0] if r is not None else M.norm(last)
            r = self._call("lm_head", [xn, E.weight, E.scales, E.biases])
            if r is None:
                r = [E.as_linear(xn)]
        logits = r[0]
        object.__setattr__(self, "last_logits", logits)  # the last position's logits, for checks
        r = self._call("logits_pick", [logits])
        if r is None:
            lse = torch.logsumexp(logits.float(), dim=-1, keepdim=True)
            lp = (logits.float() - lse.to(logits.dtype).float()).to(logits.dtype)
            tok = torch.argmax(lp, dim=-1).to(torch.int32)
            return tok, lp.float().gather(-1, tok.long()[:, None]).reshape(1)
        return r[0], r[1]
