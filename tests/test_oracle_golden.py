"""Pin the CPU oracle (oracle/qwen35_oracle.py) against fixtures produced by the installed
transformers library (tests/golden/make_golden.py): tokens, logits and states, bit for bit."""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle.qwen35_oracle import Oracle
from qwen35_b200.config import QWEN35_0P8B, TINY
from qwen35_b200.weights import make_random_weights, make_token_ids

VARIANTS = [("hf", torch.bfloat16), ("f32", torch.float32)]


@pytest.mark.parametrize("name", ["tiny_p70_g12", "tiny_p3_g6"])
@pytest.mark.parametrize("variant,state_dtype", VARIANTS)
def test_tiny_bit_exact(name, variant, state_dtype):
    g = load_golden(f"{name}_{variant}")
    w = make_random_weights(int(g["seed_weights"]), TINY)
    ids = torch.from_numpy(g["prompt_ids"])
    assert torch.equal(ids, make_token_ids(ids.numel(), int(g["seed_ids"]), TINY.vocab))
    o = Oracle(w, TINY, 4096, state_dtype=state_dtype)
    toks, logits = o.generate(ids, len(g["tokens"]))
    assert toks == g["tokens"].tolist()
    assert np.array_equal(torch.stack(logits).float().numpy(), g["logits"])
    # final states, HuggingFace layouts
    assert np.array_equal(torch.stack(o.dn_state).float().numpy(), g["dn_state"])
    assert np.array_equal(torch.stack([c[0] for c in o.conv_state]).float().numpy(), g["conv_state"])
    assert np.array_equal(torch.stack(o.k_cache).float().numpy(), g["k_cache"])
    assert np.array_equal(torch.stack(o.v_cache).float().numpy(), g["v_cache"])


@pytest.mark.parametrize("variant,state_dtype,n_steps", [("f32", torch.float32, 128), ("hf", torch.bfloat16, 20)])
def test_full_dims_bit_exact(full_weights_cpu, variant, state_dtype, n_steps):
    g = load_golden(f"qwen35_0p8b_p520_g128_{variant}")
    ids = torch.from_numpy(g["prompt_ids"])
    assert torch.equal(ids, make_token_ids(520, 7, QWEN35_0P8B.vocab))
    o = Oracle(full_weights_cpu, QWEN35_0P8B, 2048, state_dtype=state_dtype)
    toks, logits = o.generate(ids, n_steps)
    assert toks == g["tokens"][:n_steps].tolist()
    lg = torch.stack(logits).float()
    stride = int(g["logit_stride"])
    assert np.array_equal(lg[:, ::stride].numpy(), g["logits_sampled"][:n_steps])
    top = torch.topk(lg, 8, dim=-1)
    assert np.array_equal(top.values.numpy(), g["top_vals"][:n_steps])
    if n_steps == len(g["tokens"]):
        dn = torch.stack(o.dn_state).float()
        assert np.array_equal(dn[0, :, ::16, ::16].numpy(), g["dn_state_l0"])
        assert np.array_equal(dn[-1, :, ::16, ::16].numpy(), g["dn_state_last"])
        assert np.array_equal(torch.stack(o.k_cache)[:, :, -1].float().numpy(), g["k_last"])
        assert np.array_equal(torch.stack(o.v_cache)[:, :, -1].float().numpy(), g["v_last"])


def test_reference_layout_views():
    """The reference keeps the DeltaNet state value-major ([head][v][k], kernel.cu:684)."""
    w = make_random_weights(3, TINY)
    o = Oracle(w, TINY)
    o.prefill(make_token_ids(9, 1, TINY.vocab))
    ref = o.dn_states_ref_layout()
    assert ref.shape == (TINY.n_dn, TINY.dn_heads, TINY.dn_value_dim, TINY.dn_key_dim)
    assert torch.equal(ref[2, 1, 3, 5], o.dn_state[2][1, 5, 3])
    assert o.conv_ref_layout().shape == (TINY.n_dn, TINY.dn_conv_channels, 4)


def test_chunk_and_recurrent_forms_agree():
    """Prefill (chunk-64) and token-serial decode are the same recurrence up to rounding."""
    w = make_random_weights(5, TINY)
    ids = make_token_ids(150, 2, TINY.vocab)
    a = Oracle(w, TINY)
    la = a.prefill(ids)
    b = Oracle(w, TINY)
    for t in ids.tolist():
        lb = b.step(t)
    assert (la.float() - lb.float()).abs().max() < 2e-2
    sa, sb = torch.stack(a.dn_state), torch.stack(b.dn_state)
    assert (sa - sb).norm() / sa.norm() < 1e-2
