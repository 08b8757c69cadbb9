"""The reference's own CPU ground truth: HuggingFace `transformers` eager Qwen3.5 with the
pure-torch DeltaNet functions (the "PyTorch HF" arm of models/qwen35_0p8b/final_bench.py:241-304).
TEST / CPU-BASELINE INFRASTRUCTURE ONLY -- never imported by the product package.

`transformers` (5.5.0, models/qwen3_5) is a third-party dependency of the reference that is
installed in this image; nothing is copied from it.  Used by tests/golden/make_golden.py to
produce fixtures and by `bench.py --impl reference` as the timed reference arm.
"""
from __future__ import annotations

import torch

FA_NAMES = ["input_layernorm.weight", "self_attn.q_proj.weight", "self_attn.k_proj.weight",
            "self_attn.v_proj.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight",
            "self_attn.o_proj.weight", "post_attention_layernorm.weight", "mlp.gate_proj.weight",
            "mlp.up_proj.weight", "mlp.down_proj.weight"]
DN_NAMES = ["input_layernorm.weight", "linear_attn.in_proj_qkv.weight", "linear_attn.in_proj_z.weight",
            "linear_attn.in_proj_b.weight", "linear_attn.in_proj_a.weight", "linear_attn.conv1d.weight",
            "linear_attn.A_log", "linear_attn.dt_bias", "linear_attn.norm.weight",
            "linear_attn.out_proj.weight", "post_attention_layernorm.weight", "mlp.gate_proj.weight",
            "mlp.up_proj.weight", "mlp.down_proj.weight"]


def build_hf(weights: dict, d):
    """Qwen3_5ForCausalLM on CPU, bf16, eager attention, torch DeltaNet path, loaded from the
    reference-format `weights` dict (tensor order of models/qwen35_0p8b/model.py:342-380)."""
    import transformers.models.qwen3_5.modeling_qwen3_5 as M
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig

    # force the torch implementations even where fla / causal-conv1d are installed
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
    try:
        with torch.device("meta"):
            model = M.Qwen3_5ForCausalLM(cfg)
    finally:
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
    """Make the library's cache keep the DeltaNet state in f32 (it otherwise stores it in the
    dtype of the conv state, bf16).  Returns a function that undoes the patch."""
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
def greedy(model, ids: torch.Tensor, n_new: int):
    """Prompt forward + cached greedy loop, as final_bench.py:256-290.  Returns
    (tokens, stacked f32 logits of every step, cache, seconds_prefill, seconds_decode)."""
    import time
    t0 = time.perf_counter()
    out = model(input_ids=ids[None].long(), use_cache=True)
    t1 = time.perf_counter()
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
    t2 = time.perf_counter()
    return toks, torch.stack(logits).float(), pkv, t1 - t0, t2 - t1
