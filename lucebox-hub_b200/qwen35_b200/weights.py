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


# Checkpoint tensor names of one layer, in pointer order (models/qwen35_0p8b/model.py:342-380).
FA_TENSOR_NAMES = ("input_layernorm.weight", "self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                   "self_attn.q_norm.weight", "self_attn.k_norm.weight", "self_attn.o_proj.weight",
                   "post_attention_layernorm.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight")
DN_TENSOR_NAMES = ("input_layernorm.weight", "linear_attn.in_proj_qkv.weight", "linear_attn.in_proj_z.weight",
                   "linear_attn.in_proj_b.weight", "linear_attn.in_proj_a.weight", "linear_attn.conv1d.weight",
                   "linear_attn.A_log", "linear_attn.dt_bias", "linear_attn.norm.weight", "linear_attn.out_proj.weight",
                   "post_attention_layernorm.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight")
# prefixes under which the text model's tensors appear in published checkpoints (plain causal LM, multimodal wrapper)
_CHECKPOINT_PREFIXES = ("model.", "model.language_model.", "language_model.model.")


def state_dict_names(dims: Dims = QWEN35_0P8B, prefix: str = "model."):
    """(name, layer index or None, slot index or key) for every tensor of the weights dict, checkpoint naming."""
    out = [(prefix + "embed_tokens.weight", None, "embed_weight"), (prefix + "norm.weight", None, "final_norm_weight")]
    for i, lt in enumerate(dims.layer_types):
        names = FA_TENSOR_NAMES if lt == 1 else DN_TENSOR_NAMES
        out += [(f"{prefix}layers.{i}.{n}", i, s) for s, n in enumerate(names)]
    return out


def weights_to_state_dict(weights: dict, dims: Dims = QWEN35_0P8B, prefix: str = "model.") -> dict:
    """The weights dict under its checkpoint names (what `save_file` of safetensors takes)."""
    sd = {}
    for name, layer, slot in state_dict_names(dims, prefix):
        sd[name] = (weights[slot] if layer is None else weights["layer_data"][layer]["ptrs"][slot]).contiguous()
    if weights["lm_head_weight"] is not weights["embed_weight"]:
        sd["lm_head.weight"] = weights["lm_head_weight"].contiguous()
    return sd


def load_safetensors_weights(path: str, dims: Dims = QWEN35_0P8B, device="cpu") -> dict:
    """Build the weights dict from a HuggingFace checkpoint directory (`*.safetensors`, sharded or not) or a single
    `.safetensors` file: the file-reading half of the reference's `load_weights` (models/qwen35_0p8b/model.py:314-407;
    the reference goes through `AutoModelForCausalLM.from_pretrained`, which needs the network and a GPU-side model
    copy; this reads the tensors directly).  Tensors are taken as stored (bf16 expected), shapes are checked, the LM
    head is tied to the embedding when the checkpoint has no `lm_head.weight`."""
    import glob
    import os

    from safetensors import safe_open

    files = [path] if os.path.isfile(path) else sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no .safetensors file under {path}")
    where = {}
    for f in files:
        with safe_open(f, framework="pt", device="cpu") as sf:
            for k in sf.keys():
                where[k] = f
    prefix = next((p for p in _CHECKPOINT_PREFIXES if p + "embed_tokens.weight" in where), None)
    if prefix is None:
        raise KeyError("embed_tokens.weight not found under any known prefix: " + ", ".join(_CHECKPOINT_PREFIXES))
    handles = {f: safe_open(f, framework="pt", device="cpu") for f in files}

    def get(name, shape=None):
        if name not in where:
            raise KeyError(f"tensor {name} missing from the checkpoint")
        t = handles[where[name]].get_tensor(name)
        if t.dtype != torch.bfloat16:
            t = t.to(torch.bfloat16)
        if shape is not None and tuple(t.shape) != tuple(shape):
            raise ValueError(f"{name}: shape {tuple(t.shape)}, expected {tuple(shape)}")
        return t.contiguous().to(device)

    d = dims
    fa_shapes = ((d.hidden,), (2 * d.fa_q_heads * d.fa_head_dim, d.hidden), (d.fa_kv_heads * d.fa_head_dim, d.hidden),
                 (d.fa_kv_heads * d.fa_head_dim, d.hidden), (d.fa_head_dim,), (d.fa_head_dim,),
                 (d.hidden, d.fa_q_heads * d.fa_head_dim), (d.hidden,), (d.intermediate, d.hidden), (d.intermediate, d.hidden),
                 (d.hidden, d.intermediate))
    dn_v = d.dn_heads * d.dn_value_dim
    dn_shapes = ((d.hidden,), (d.dn_conv_channels, d.hidden), (dn_v, d.hidden), (d.dn_heads, d.hidden), (d.dn_heads, d.hidden),
                 (d.dn_conv_channels, 1, d.dn_conv_kernel), (d.dn_heads,), (d.dn_heads,), (d.dn_value_dim,), (d.hidden, dn_v),
                 (d.hidden,), (d.intermediate, d.hidden), (d.intermediate, d.hidden), (d.hidden, d.intermediate))
    layer_data = []
    for i, lt in enumerate(d.layer_types):
        names, shapes = (FA_TENSOR_NAMES, fa_shapes) if lt == 1 else (DN_TENSOR_NAMES, dn_shapes)
        layer_data.append({"type": int(lt), "ptrs": [get(f"{prefix}layers.{i}.{n}", s) for n, s in zip(names, shapes)]})
    embed = get(prefix + "embed_tokens.weight", (d.vocab, d.hidden))
    lm = get("lm_head.weight", (d.vocab, d.hidden)) if "lm_head.weight" in where else embed
    return {"embed_weight": embed, "final_norm_weight": get(prefix + "norm.weight", (d.hidden,)), "lm_head_weight": lm,
            "layer_data": layer_data}
