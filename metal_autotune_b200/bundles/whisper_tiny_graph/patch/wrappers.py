"""Graph-backend region wrappers (autotuner_runtime/graph.py): the tiny
GELU-MLP and the Whisper encoder served by their traced aten graphs with
every region occurrence substituted by its kernel, instead of by a
hand-written replay of the forward (the reference's GraphWrapper bundles,
autotuner_runtime/graph.py:306-502).

What each class serves is recorded per call signature in graph_variants.json
beside this file (written by `python -m metal_autotune_b200.bundles`): the
rules in the order they rewrite, each with its pattern's input shapes, the
number of occurrences it must replace and its anchors. A signature that
matches no variant, or whose graph no longer holds exactly the recorded
occurrences, runs the wrapped module's own forward (with MT_STRICT_REGIONS=1
it raises instead).
"""
import json
from pathlib import Path

from metal_autotune_b200.autotuner_runtime.graph import GraphWrapper


def _variants(name: str) -> tuple:
    f = Path(__file__).with_name("graph_variants.json")
    return tuple(json.loads(f.read_text()).get(name, ())) if f.exists() else ()


class G_tiny_mlp(GraphWrapper):
    KERNEL_IDS = ["linear_gelu_f32", "linear_f32"]
    GRAPH_VARIANTS = _variants("G_tiny_mlp")


class G_whisper_encoder(GraphWrapper):
    KERNEL_IDS = ["conv1_gelu", "conv2_gelu", "pos_add", "fc1_gelu", "fc2_residual", "out_proj_residual",
                  "attention", "linear_bias", "linear_nobias", "layer_norm"]
    GRAPH_VARIANTS = _variants("G_whisper_encoder")
