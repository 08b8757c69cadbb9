"""CPU checks of the DFlash draft oracle: its plain mathematical form (no intermediate roundings) against an
independently written implementation (complex-number rotary embedding, torch's scaled_dot_product_attention with
repeated kv heads), the size of the bf16 rounding effect, and the edge cases the GPU tests rely on."""
import math
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "lucebox-hub_b200"))

from oracle.dflash_draft_oracle import draft_forward  # noqa: E402
from qwen35_b200.dflash_draft import DraftDims, make_random_draft_weights  # noqa: E402


def _independent(D, w, noise, thc):
    def rms(x, wt):
        return x / torch.sqrt(x.pow(2).mean(-1, keepdim=True) + D.eps) * wt

    def rope(x, pos):                                  # x [rows, heads, hd]; NEOX: element i pairs with i + hd/2
        hd = x.shape[-1]
        inv = D.rope_theta ** (-torch.arange(0, hd, 2, dtype=torch.float64) / hd)
        ang = pos.double()[:, None] * inv[None, :]
        z = torch.complex(x[..., : hd // 2].double(), x[..., hd // 2:].double()) * torch.polar(torch.ones_like(ang), ang)[:, None, :]
        return torch.cat([z.real, z.imag], -1).float()

    ctx, q = thc.shape[0], D.q_len
    feat = rms(thc.float() @ w["fc"].float().t(), w["hidden_norm"])
    h = noise.float()
    rep = D.n_heads // D.n_kv_heads
    for L in w["layers"]:
        hn = rms(h, L["attn_norm"])
        wk, wv = L["wkv"].float()[: D.kv_dim], L["wkv"].float()[D.kv_dim:]
        allrows = torch.cat([feat, hn], 0)
        Q = rope(rms((hn @ L["wq"].float().t()).view(q, D.n_heads, D.head_dim), L["q_norm"]), torch.arange(ctx, ctx + q))
        K = rope(rms((allrows @ wk.t()).view(ctx + q, D.n_kv_heads, D.head_dim), L["k_norm"]), torch.arange(ctx + q))
        V = (allrows @ wv.t()).view(ctx + q, D.n_kv_heads, D.head_dim)
        o = torch.nn.functional.scaled_dot_product_attention(Q.transpose(0, 1)[None], K.transpose(0, 1).repeat_interleave(rep, 0)[None],
                                                             V.transpose(0, 1).repeat_interleave(rep, 0)[None], is_causal=False)
        h = h + o[0].transpose(0, 1).reshape(q, D.q_dim) @ L["wo"].float().t()
        hf = rms(h, L["ffn_norm"])
        wg, wu = L["w_gate_up"].float()[: D.inter], L["w_gate_up"].float()[D.inter:]
        h = h + (torch.nn.functional.silu(hf @ wg.t()) * (hf @ wu.t())) @ L["w_down"].float().t()
    return rms(h, w["out_norm"])


def _case(ctx, seed=0):
    D = DraftDims(hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, inter=512, q_len=8)
    w = make_random_draft_weights(D, seed)
    g = torch.Generator().manual_seed(seed + 1)
    noise = torch.randn(D.q_len, D.hidden, generator=g).bfloat16()
    thc = torch.randn(ctx, D.n_target_layers * D.hidden, generator=g).bfloat16()
    return D, w, noise, thc


def test_oracle_equals_independent_implementation():
    for ctx in (1, 37, 130):
        D, w, noise, thc = _case(ctx, ctx)
        a = draft_forward(D, w, noise, thc, rounding=False)
        b = _independent(D, w, noise, thc)
        assert float((a - b).abs().max()) <= 2e-4 * max(1.0, float(b.abs().max()))


def test_bf16_rounding_points_move_the_result_by_a_few_bf16_steps_only():
    D, w, noise, thc = _case(64, 5)
    exact = draft_forward(D, w, noise, thc, rounding=False)
    rounded = draft_forward(D, w, noise, thc).float()
    rel = float((rounded - exact).abs().max() / exact.abs().max())
    assert 0.0 < rel < 0.05


def test_empty_context_and_head():
    D, w, noise, _ = _case(1, 9)
    out = draft_forward(D, w, noise, None)
    assert out.shape == (D.q_len, D.hidden) and out.dtype == torch.bfloat16 and bool(torch.isfinite(out.float()).all())
    head = (torch.randn(96, D.hidden, generator=torch.Generator().manual_seed(2)) * 0.05).bfloat16()
    out2, logits = draft_forward(D, w, noise, None, lm_head=head)
    assert torch.equal(out, out2) and logits.shape == (D.q_len, 96)
    # position 0 is not rotated: with a single noise row as the only key, attention returns that row's value
    assert math.isfinite(float(logits.float().abs().max()))
