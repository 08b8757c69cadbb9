"""Seeded random-init weights in the reference's `weights` dict format.

The reference builds this dict from a HuggingFace checkpoint
(models/qwen35_0p8b/model.py:314-407): `embed_weight`, `final_norm_weight`,
`lm_head_weight` (tied to the embedding, model.py:384) and `layer_data`, a list of
`{"type": 0|1, "ptrs": [tensor, ...]}` with 14 tensors for a DeltaNet layer and 11
for a full-attention layer, in the order of model.py:342-380.  No checkpoint can be
downloaded where this code runs, so the same structure is filled from a counter
based generator (numpy Philox, float64 normals rounded once to bf16) which gives
identical bits on every machine.
"""
from __future__ import annotations

import numpy as np
import torch

from .config import Dims, QWEN35_0P8B

# Pointer slots of one layer record (models/qwen35_0p8b/kernel.cu:77-115).
FA_SLOTS = ("input_layernorm", "q_proj", "k_proj", "v_proj", "q_norm", "k_norm", "o_proj",
            "post_attention_layernorm", "gate_proj", "up_proj", "down_proj")
DN_SLOTS = ("input_layernorm", "in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "conv1d",
            "A_log", "dt_bias", "norm", "out_proj", "post_attention_layernorm",
            "gate_proj", "up_proj", "down_proj")


def _bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16)


class _Gen:
    def __init__(self, seed: int):
        self.rng = np.random.Generator(np.random.Philox(seed))

    def normal(self, shape, std=0.02, mean=0.0):
        return _bf16(self.rng.standard_normal(shape) * std + mean)

    def uniform_log(self, n, lo, hi):
        return _bf16(np.log(self.rng.uniform(lo, hi, n)))


def make_random_weights(seed: int = 1234, dims: Dims = QWEN35_0P8B, device="cpu") -> dict:
    """All matrices ~ N(0, 0.02); `(1+w)` norm weights ~ N(0, 0.02); the DeltaNet gated
    norm weight and `dt_bias` ~ N(1, 0.02); `A_log` = log U(0.5, 16)."""
    g = _Gen(seed)
    d = dims
    embed = g.normal((d.vocab, d.hidden))
    layer_data = []
    for lt in d.layer_types:
        if lt == 1:
            ptrs = [
                g.normal((d.hidden,)),
                g.normal((d.fa_qproj_size, d.hidden)),
                g.normal((d.fa_kv_size, d.hidden)),
                g.normal((d.fa_kv_size, d.hidden)),
                g.normal((d.fa_head_dim,)),
                g.normal((d.fa_head_dim,)),
                g.normal((d.hidden, d.fa_q_size)),
                g.normal((d.hidden,)),
                g.normal((d.intermediate, d.hidden)),
                g.normal((d.intermediate, d.hidden)),
                g.normal((d.hidden, d.intermediate)),
            ]
        else:
            ptrs = [
                g.normal((d.hidden,)),
                g.normal((d.dn_conv_channels, d.hidden)),
                g.normal((d.dn_v_size, d.hidden)),
                g.normal((d.dn_heads, d.hidden)),
                g.normal((d.dn_heads, d.hidden)),
                g.normal((d.dn_conv_channels, 1, d.dn_conv_kernel)),
                g.uniform_log(d.dn_heads, 0.5, 16.0),
                g.normal((d.dn_heads,), mean=1.0),
                g.normal((d.dn_value_dim,), mean=1.0),
                g.normal((d.hidden, d.dn_v_size)),
                g.normal((d.hidden,)),
                g.normal((d.intermediate, d.hidden)),
                g.normal((d.intermediate, d.hidden)),
                g.normal((d.hidden, d.intermediate)),
            ]
        layer_data.append({"type": lt, "ptrs": [p.to(device).contiguous() for p in ptrs]})
    final_norm = g.normal((d.hidden,))
    embed = embed.to(device).contiguous()
    return {
        "embed_weight": embed,
        "final_norm_weight": final_norm.to(device).contiguous(),
        "lm_head_weight": embed,
        "layer_data": layer_data,
    }


def make_token_ids(n: int, seed: int = 7, vocab: int = QWEN35_0P8B.vocab) -> torch.Tensor:
    """Uniform random prompt ids (stand-in for the reference's English seed prompt,
    models/qwen35_0p8b/final_bench.py:52-62), int32."""
    rng = np.random.Generator(np.random.Philox(seed))
    return torch.from_numpy(rng.integers(0, vocab, size=n, dtype=np.int64).astype(np.int32))


def weights_to(weights: dict, device) -> dict:
    """Copy a weights dict to `device`, keeping the embedding/LM-head tie."""
    embed = weights["embed_weight"].to(device)
    tied = weights["lm_head_weight"] is weights["embed_weight"]
    return {
        "embed_weight": embed,
        "final_norm_weight": weights["final_norm_weight"].to(device),
        "lm_head_weight": embed if tied else weights["lm_head_weight"].to(device),
        "layer_data": [{"type": ld["type"], "ptrs": [p.to(device) for p in ld["ptrs"]]}
                       for ld in weights["layer_data"]],
    }
