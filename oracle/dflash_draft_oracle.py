"""TEST INFRASTRUCTURE ONLY (imported by tests/ and bench.py's CPU-baseline leg; never by the product).

CPU restatement of the DFlash draft forward, following build_draft_graph
(models/qwen35_27b/src/qwen3_dflash_graph.cpp:38-166) op by op:

    :59-62   target_feat = rms_norm(fc @ target_hidden_cat) * hidden_norm
    :71-72   hn = rms_norm(h) * attn_norm
    :76-79   Q = wq @ hn, per-head rms_norm * q_norm
    :83-98   K, V = wk / wv @ [target_feat ; hn]; per-head rms_norm(K) * k_norm
    :104-110 NEOX RoPE (pairs i, i + head_dim/2; theta_i = pos * base^(-2i/head_dim)), Q at ctx_len + i, K at 0..total_k-1
    :126-128 non-causal softmax(Q K^T / sqrt(head_dim)) V, GQA by head grouping
    :135-136 h += wo @ attn
    :139-152 h += w_down @ (silu(w_gate @ hf) * (w_up @ hf)), hf = rms_norm(h) * ffn_norm
    :156-157 out = rms_norm(h) * out_norm

Parity unpinned: the arithmetic of these ops lives in the ggml fork the reference pulls in as a submodule (absent here, no
commit pin recoverable) and the Python reference the file names (dflash_reference.py) is not in the tree, so there is no
golden vector to pin against.  What is restated is the published meaning of each op.  Rounding points are this build's
convention (every module output rounded once to bf16, f32 accumulation inside), the same as on the other paths:
GEMM outputs, the residual epilogue bf16(bf16(acc) + r), the SwiGLU epilogue bf16(bf16(silu(bf16 g)) * bf16 u), norms,
rotated Q / K, attention output.  Softmax probabilities are kept in f32 here (the kernel rounds them to bf16 relative
to a chunk-local maximum); the tests' tolerance covers that difference."""
import math

import torch


def _bf(x):
    return x.bfloat16().float()


def _rms(x, w, eps, _bf=_bf):
    return _bf(x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps) * w)


def _norm_rope(x, w, eps, base, pos, _bf=_bf):
    """x f32 [rows, heads, hd] (bf16 values), pos int64 [rows] -> bf16-rounded f32."""
    hd = x.shape[-1]
    y = x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps) * w
    i = torch.arange(hd // 2, dtype=torch.float64)
    theta = pos.double()[:, None] * torch.pow(torch.tensor(base, dtype=torch.float64), -2.0 * i / hd)[None, :]
    cs, sn = torch.cos(theta).float()[:, None, :], torch.sin(theta).float()[:, None, :]
    y0, y1 = y[..., : hd // 2], y[..., hd // 2:]
    return _bf(torch.cat([y0 * cs - y1 * sn, y0 * sn + y1 * cs], dim=-1))


def draft_forward(dims, w, noise_embed, target_hidden_cat, lm_head=None, trace=None, rounding=True):
    """dims: qwen35_b200.dflash_draft.DraftDims; w: CPU weights from make_random_draft_weights; tensors bf16 on the CPU.
    Returns hidden_out bf16 [q_len, hidden] (and logits bf16 when lm_head, a dense bf16-valued matrix, is given).
    rounding=False drops every intermediate bf16 rounding and returns f32: the plain mathematical function, which the
    CPU tests compare with an independently written implementation."""
    bf = _bf if rounding else (lambda x: x)
    D = dims
    q, hd, gqa = D.q_len, D.head_dim, D.n_heads // D.n_kv_heads
    ctx = 0 if target_hidden_cat is None else target_hidden_cat.shape[0]
    T = ctx + q
    if ctx:
        feat = _rms(bf(target_hidden_cat.float() @ w["fc"].float().t()), w["hidden_norm"], D.eps, bf)
    else:
        feat = torch.zeros(0, D.hidden)
    h = noise_embed.float()
    pos_q, pos_k = torch.arange(ctx, T), torch.arange(T)
    scale = 1.0 / math.sqrt(hd)
    for L in w["layers"]:
        hn = _rms(h, L["attn_norm"], D.eps, bf)
        X = torch.cat([feat, hn], dim=0)
        Q = bf(hn @ L["wq"].float().t()).view(q, D.n_heads, hd)
        KV = bf(X @ L["wkv"].float().t())
        K = KV[:, : D.kv_dim].reshape(T, D.n_kv_heads, hd)
        V = KV[:, D.kv_dim:].reshape(T, D.n_kv_heads, hd)
        Q = _norm_rope(Q, L["q_norm"], D.eps, D.rope_theta, pos_q, bf)
        K = _norm_rope(K, L["k_norm"], D.eps, D.rope_theta, pos_k, bf)
        attn = torch.empty(q, D.n_heads, hd)
        for head in range(D.n_heads):
            kvh = head // gqa
            s = (Q[:, head] @ K[:, kvh].t()) * scale
            attn[:, head] = torch.softmax(s, dim=-1) @ V[:, kvh]
        attn = bf(attn).view(q, D.q_dim)
        h = bf(bf(attn @ L["wo"].float().t()) + h)
        hf = _rms(h, L["ffn_norm"], D.eps, bf)
        gu = hf @ L["w_gate_up"].float().t()
        g, u = bf(gu[:, : D.inter]), bf(gu[:, D.inter:])
        act = bf(bf(g * torch.sigmoid(g)) * u)
        h = bf(bf(act @ L["w_down"].float().t()) + h)
        if trace is not None:
            trace.append(h.bfloat16())
    out = _rms(h, w["out_norm"], D.eps, bf)
    if rounding:
        out = out.bfloat16()
    if lm_head is None:
        return out
    logits = bf(out.float() @ lm_head.float().t())
    return out, (logits.bfloat16() if rounding else logits)
