"""Generate the golden fixtures in this directory from the installed `transformers`.

The reference's ground truth for its Qwen3.5 kernels is HuggingFace eager PyTorch with the
pure-torch DeltaNet functions (models/qwen35_0p8b/final_bench.py:241-304).  This script
builds `Qwen3_5ForCausalLM` (transformers 5.5.0) on CPU with eager attention and the torch
DeltaNet path, loads the seeded random-init weights of `qwen35_b200.weights`, runs a prompt
prefill followed by greedy decode, and stores tokens, logits and final states.

Two variants are written per configuration:
  *_hf.npz   the unmodified library.  Its cache stores the DeltaNet state in the dtype of
             the conv state, i.e. rounds it to bf16 after every call.
  *_f32.npz  the same run with `LinearAttentionLayer.lazy_initialization` patched so the
             state buffer keeps f32 -- what the reference kernels do (model.py:538,
             kernel.cu:684-695) and what the CUDA path is compared against.

Run from the repository root:  python tests/golden/make_golden.py [tiny|full|all]
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "lucebox-hub_b200"))

from qwen35_b200.config import QWEN35_0P8B, TINY  # noqa: E402
from qwen35_b200.weights import make_random_weights, make_token_ids  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))

FA_NAMES = ["input_layernorm.weight", "self_attn.q_proj.weight", "self_attn.k_proj.weight",
            "self_attn.v_proj.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight",
            "self_attn.o_proj.weight", "post_attention_layernorm.weight", "mlp.gate_proj.weight",
            "mlp.up_proj.weight", "mlp.down_proj.weight"]
DN_NAMES = ["input_layernorm.weight", "linear_attn.in_proj_qkv.weight", "linear_attn.in_proj_z.weight",
            "linear_attn.in_proj_b.weight", "linear_attn.in_proj_a.weight", "linear_attn.conv1d.weight",
            "linear_attn.A_log", "linear_attn.dt_bias", "linear_attn.norm.weight",
            "linear_attn.out_proj.weight", "post_attention_layernorm.weight", "mlp.gate_proj.weight",
            "mlp.up_proj.weight", "mlp.down_proj.weight"]


def build_hf(weights, d):
    import transformers.models.qwen3_5.modeling_qwen3_5 as M
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig

    for n in ("chunk_gated_delta_rule", "fused_recurrent_gated_delta_rule", "FusedRMSNormGated",
              "causal_conv1d_fn", "causal_conv1d_update"):
        setattr(M, n, None)
    cfg = Qwen3_5TextConfig(
        vocab_size=d.vocab, hidden_size=d.hidden, intermediate_size=d.intermediate,
        num_hidden_layers=d.num_layers, num_attention_heads=d.fa_q_heads,
        num_key_value_heads=d.fa_kv_heads, head_dim=d.fa_head_dim,
        linear_key_head_dim=d.dn_key_dim, linear_value_head_dim=d.dn_value_dim,
        linear_num_key_heads=d.dn_k_heads, linear_num_value_heads=d.dn_heads,
        linear_conv_kernel_dim=d.dn_conv_kernel, tie_word_embeddings=True,
        max_position_embeddings=8192,
        rope_parameters={"rope_type": "default", "rope_theta": d.rope_theta,
                         "partial_rotary_factor": d.fa_rotary_dim / d.fa_head_dim,
                         "mrope_section": [11, 11, 10]})
    cfg._attn_implementation = "eager"
    torch.set_default_dtype(torch.bfloat16)
    with torch.device("meta"):
        model = M.Qwen3_5ForCausalLM(cfg)
    torch.set_default_dtype(torch.float32)
    model = model.to_empty(device="cpu")
    sd = {"model.embed_tokens.weight": weights["embed_weight"],
          "lm_head.weight": weights["lm_head_weight"],
          "model.norm.weight": weights["final_norm_weight"]}
    for i, ld in enumerate(weights["layer_data"]):
        names = FA_NAMES if ld["type"] == 1 else DN_NAMES
        for n, t in zip(names, ld["ptrs"]):
            sd[f"model.layers.{i}.{n}"] = t
    res = model.load_state_dict(sd, strict=False, assign=True)
    assert not res.missing_keys and not res.unexpected_keys, res
    model.model.rotary_emb = M.Qwen3_5TextRotaryEmbedding(cfg)   # non-persistent inv_freq buffer
    return model.eval()


def patch_cache_f32():
    from transformers import cache_utils
    orig = cache_utils.LinearAttentionLayer.lazy_initialization

    def lazy(self, conv_states=None, recurrent_states=None):
        orig(self, conv_states=conv_states, recurrent_states=None)
        if recurrent_states is not None:
            self.recurrent_states = torch.zeros_like(recurrent_states)
            self.is_recurrent_states_initialized = True

    cache_utils.LinearAttentionLayer.lazy_initialization = lazy
    return lambda: setattr(cache_utils.LinearAttentionLayer, "lazy_initialization", orig)


@torch.no_grad()
def run(model, ids, n_new):
    out = model(input_ids=ids[None].long(), use_cache=True)
    pkv = out.past_key_values
    logits = [out.logits[0, -1]]
    toks = []
    for i in range(n_new):
        t = int(logits[-1].argmax())
        toks.append(t)
        if i == n_new - 1:
            break
        out = model(input_ids=torch.tensor([[t]]), past_key_values=pkv, use_cache=True)
        logits.append(out.logits[0, -1])
    return toks, torch.stack(logits).float(), pkv


def states(pkv, d):
    dn, conv, kc, vc = [], [], [], []
    for lt, layer in zip(d.layer_types, pkv.layers):
        if lt == 0:
            dn.append(layer.recurrent_states[0].float())
            conv.append(layer.conv_states[0].float())
        else:
            kc.append(layer.keys[0].float())
            vc.append(layer.values[0].float())
    return torch.stack(dn), torch.stack(conv), torch.stack(kc), torch.stack(vc)


def make(name, d, seed_w, seed_ids, n_prompt, n_new, full_logits):
    w = make_random_weights(seed_w, d)
    ids = make_token_ids(n_prompt, seed_ids, d.vocab)
    model = build_hf(w, d)
    for variant in ("hf", "f32"):
        undo = patch_cache_f32() if variant == "f32" else (lambda: None)
        toks, logits, pkv = run(model, ids, n_new)
        undo()
        dn, conv, kc, vc = states(pkv, d)
        top = torch.topk(logits, 8, dim=-1)
        rec = dict(seed_weights=seed_w, seed_ids=seed_ids, prompt_ids=ids.numpy(),
                   tokens=np.array(toks, dtype=np.int32),
                   top_vals=top.values.numpy(), top_idx=top.indices.numpy().astype(np.int32))
        if full_logits:
            rec.update(logits=logits.numpy(), dn_state=dn.numpy(), conv_state=conv.numpy(),
                       k_cache=kc.numpy(), v_cache=vc.numpy())
        else:
            # samples only: every 97th logit of every step, a few state rows, the newest K/V rows
            rec.update(logit_stride=97, logits_sampled=logits[:, ::97].numpy(),
                       dn_state_l0=dn[0, :, ::16, ::16].numpy(), dn_state_last=dn[-1, :, ::16, ::16].numpy(),
                       dn_state_norms=dn.flatten(2).norm(dim=-1).numpy(),
                       conv_state_sampled=conv[:, ::64].numpy(),
                       k_last=kc[:, :, -1].numpy(), v_last=vc[:, :, -1].numpy())
        path = os.path.join(HERE, f"{name}_{variant}.npz")
        np.savez_compressed(path, **rec)
        print(path, os.path.getsize(path), "bytes; tokens[:8] =", toks[:8])


if __name__ == "__main__":
    which = sys.argv[1] if len(sys.argv) > 1 else "all"
    if which in ("tiny", "all"):
        make("tiny_p70_g12", TINY, 1234, 7, 70, 12, True)
        make("tiny_p3_g6", TINY, 99, 5, 3, 6, True)       # prompt shorter than the conv window
    if which in ("full", "all"):
        make("qwen35_0p8b_p520_g128", QWEN35_0P8B, 1234, 7, 520, 128, False)
