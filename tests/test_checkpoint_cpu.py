"""CPU: checkpoint ingestion.  A safetensors file written under the checkpoint tensor names loads back into the very
same weights dict (names, pointer order, shapes, LM-head tie); wrong shapes and missing tensors are refused."""
import os

import pytest
import torch


def _tiny():
    from qwen35_b200.config import TINY
    from qwen35_b200.weights import make_random_weights
    return TINY, make_random_weights(5, TINY)


@pytest.mark.parametrize("prefix", ["model.", "model.language_model."])
def test_safetensors_round_trip(tmp_path, prefix):
    from safetensors.torch import save_file
    from qwen35_b200.weights import load_safetensors_weights, weights_to_state_dict
    D, w = _tiny()
    sd = weights_to_state_dict(w, D, prefix)
    # two shards, as published checkpoints are
    keys = sorted(sd)
    save_file({k: sd[k] for k in keys[::2]}, str(tmp_path / "model-00001-of-00002.safetensors"))
    save_file({k: sd[k] for k in keys[1::2]}, str(tmp_path / "model-00002-of-00002.safetensors"))
    got = load_safetensors_weights(str(tmp_path), D)
    assert got["lm_head_weight"] is got["embed_weight"]                  # tied: the checkpoint has no lm_head.weight
    assert torch.equal(got["embed_weight"], w["embed_weight"]) and torch.equal(got["final_norm_weight"], w["final_norm_weight"])
    for a, b in zip(got["layer_data"], w["layer_data"]):
        assert a["type"] == b["type"] and len(a["ptrs"]) == len(b["ptrs"])
        for x, y in zip(a["ptrs"], b["ptrs"]):
            assert x.dtype == torch.bfloat16 and x.shape == y.shape and torch.equal(x, y)


def test_safetensors_names_match_the_hf_module():
    """The names are those of transformers' Qwen3_5ForCausalLM state dict."""
    from oracle.hf_reference import build_hf
    from qwen35_b200.weights import state_dict_names
    D, w = _tiny()
    hf_names = set(build_hf(w, D).state_dict().keys())
    ours = {n for n, _, _ in state_dict_names(D)}
    assert ours <= hf_names and hf_names - ours <= {"lm_head.weight"}


def test_safetensors_rejects_bad_checkpoints(tmp_path):
    from safetensors.torch import save_file
    from qwen35_b200.weights import load_safetensors_weights, weights_to_state_dict
    D, w = _tiny()
    sd = weights_to_state_dict(w, D)
    bad = dict(sd); bad["model.layers.0.mlp.up_proj.weight"] = bad["model.layers.0.mlp.up_proj.weight"][:-1].contiguous()
    save_file(bad, str(tmp_path / "a.safetensors"))
    with pytest.raises(ValueError):
        load_safetensors_weights(str(tmp_path / "a.safetensors"), D)
    missing = dict(sd); del missing["model.layers.1.input_layernorm.weight"]
    save_file(missing, str(tmp_path / "b.safetensors"))
    with pytest.raises(KeyError):
        load_safetensors_weights(str(tmp_path / "b.safetensors"), D)
    with pytest.raises(FileNotFoundError):
        load_safetensors_weights(str(tmp_path / "nothing_here"), D)
