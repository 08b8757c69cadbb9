"""CPU oracle for the Qwen3.5 hybrid forward path.  TEST INFRASTRUCTURE ONLY.

Nothing in the product package may import this file; it is used by `tests/`, by
`__graft_entry__.smoke()` and by the `cpu_baseline` / `--impl reference` legs of
`bench.py` as the checker and the timed CPU baseline.

What it restates.  The reference declares HuggingFace eager PyTorch with the
pure-torch DeltaNet functions as the ground truth of its kernels
(models/qwen35_0p8b/final_bench.py:241-304, README "PyTorch HF" rows), and its
CUDA kernels implement that network:

  * decode megakernel           models/qwen35_0p8b/kernel.cu:409-741 (layer bodies),
                                 :747-814 (LM head arg-max)
  * batched prefill             models/qwen35_0p8b/prefill.cu:1158-1464
  * weight record order         models/qwen35_0p8b/model.py:342-380

This file restates that network as plain functions over the reference's `weights`
dict, with the rounding points of a bf16 HuggingFace model (every linear returns
bf16, norms compute in f32 and round once, the DeltaNet recurrence runs in f32).
Where the reference's decode kernel and its prefill kernel disagree -- decode reads
the un-decayed state, kernel.cu:684-695, prefill decays first, prefill.cu:508-522 --
the prefill/HuggingFace form is followed.

Pinning.  `tests/golden/make_golden.py` runs the installed `transformers`
(5.5.0, models/qwen3_5, eager attention, torch DeltaNet path) on the same seeded
weights and stores tokens / logits / states; `tests/test_oracle_golden.py` checks
this file against those fixtures bit for bit.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


EXACT_LINEAR = False      # True: every projection is evaluated exactly (f64 sums) and rounded ONCE to the activation dtype


def f64_to_bf16_once(x: torch.Tensor) -> torch.Tensor:
    """float64 -> bfloat16 with a single round-to-nearest-even: first to f32 with round-to-odd (truncate toward zero, set
    the last bit when anything was lost), after which the second rounding to 8 bits cannot double-round."""
    y = x.to(torch.float32)
    y64 = y.double()
    over = y64.abs() > x.abs()
    y = torch.where(over, torch.nextafter(y, torch.zeros_like(y)), y)
    inexact = y.double() != x
    bits = y.view(torch.int32)
    bits = torch.where(inexact, bits | 1, bits)
    return bits.view(torch.float32).to(torch.bfloat16)


NVFP4_LINEAR = None       # optional {id(weight): dequantised f32 copy}: those projections are taken on NVFP4 operands (below)


def fake_quant_nvfp4_rows(x: torch.Tensor) -> torch.Tensor:
    """The values a row-major activation matrix has after quantisation to NVFP4 in the tensor-core layout
    (16-element blocks along K, UE4M3 scale = sat_rn(max(amax/6, 2^-28)), elements divided by the decoded scale and rounded
    to E2M1 to nearest even; the reference quantises prompt activations this way, prefill.cu:1210-1262 with the kernel of
    kernel_gb10_nvfp4.cu:1366-1430), as f32."""
    import numpy as np
    from . import nvfp4_ref as nv
    a = x.float().numpy().astype(np.float32)
    rows, cols = a.shape
    g = a.reshape(rows, cols // 16, 16)
    amax = np.abs(g).max(axis=-1)
    scale_f = np.maximum(amax * np.float32(1.0 / 6.0), np.float32(2.0 ** -28)).astype(np.float32)
    dec = nv.e4m3_decode(nv.e4m3_encode(scale_f))
    with np.errstate(divide="ignore"):
        inv = np.where(dec > 0, np.float32(1.0) / dec, np.float32(0.0)).astype(np.float32)
    codes = nv.e2m1_rne((g * inv[..., None]).astype(np.float32))
    vals = nv.E2M1_VALUES[codes & 7] * np.where(codes & 8, np.float32(-1.0), np.float32(1.0))
    return torch.from_numpy((vals * dec[..., None]).astype(np.float32).reshape(rows, cols))


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Projection with f32 accumulation and one rounding to the activation dtype.  bf16 weights go through
    F.linear (what a bf16 HuggingFace model does).  f32 weights are used for the NVFP4 variant, whose dequantised
    values (E2M1 code x fp16 or E4M3 scale) are exact in f32 but not in bf16 (kernel_gb10_nvfp4.cu:521-545).
    With EXACT_LINEAR the sum is taken in f64 (products of bf16 values are exact there and a 3584-term sum loses
    nothing that matters at 2^-53) and rounded once: the value every f32 summation order approximates."""
    if NVFP4_LINEAR is not None and id(w) in NVFP4_LINEAR:
        # block-scaled FP4 GEMM: both operands on the E2M1 x E4M3 grid, products and sums exact in f64, one rounding
        xq = fake_quant_nvfp4_rows(x.reshape(-1, x.shape[-1]))
        return f64_to_bf16_once(F.linear(xq.double(), NVFP4_LINEAR[id(w)].double())).reshape(*x.shape[:-1], -1).to(x.dtype)
    if EXACT_LINEAR and x.dtype == torch.bfloat16:
        return f64_to_bf16_once(F.linear(x.double(), w.double()))
    if w.dtype == x.dtype:
        return F.linear(x, w)
    return F.linear(x.float(), w.float()).to(x.dtype)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """x * rsqrt(mean x^2 + eps) * (1 + w), f32 math, one rounding to x.dtype
    (kernel.cu:173-260, `(1+w)` at :212)."""
    xf = x.float()
    out = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    out = out * (1.0 + w.float())
    return out.type_as(x)


def gated_rmsnorm(x: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """DeltaNet output norm: normalise in f32, round, multiply by w (not 1+w), times
    silu(z) (kernel.cu:697-712, plain `w` at :708)."""
    dt = x.dtype
    xf = x.to(torch.float32)
    var = xf.pow(2).mean(-1, keepdim=True)
    xf = xf * torch.rsqrt(var + eps)
    out = w * xf.to(dt)
    out = out * F.silu(z.to(torch.float32))
    return out.to(dt)


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """x * rsqrt(sum x^2 + eps) in the dtype of x (kernel.cu:646-660)."""
    inv = torch.rsqrt((x * x).sum(dim=-1, keepdim=True) + eps)
    return x * inv


def rope_tables(positions: torch.Tensor, rotary_dim: int, theta: float, dtype) -> tuple:
    """cos/sin [S, rotary_dim] rounded to `dtype`; frequencies 1/theta^(2i/rotary_dim)
    (kernel.cu:483-503; prefill.cu:597-691 uses a precomputed inv-freq table)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, rotary_dim, 2, dtype=torch.int64).to(torch.float) / rotary_dim))
    freqs = (inv_freq[None, :, None].float() @ positions[None, None, :].float()).transpose(1, 2)[0]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [heads, S, head_dim]; rotate the first `rotary_dim` dims, pairs (i, i+rd/2)."""
    rd = cos.shape[-1]
    xr, xp = x[..., :rd], x[..., rd:]
    x1, x2 = xr[..., : rd // 2], xr[..., rd // 2:]
    rot = torch.cat((-x2, x1), dim=-1)
    return torch.cat([(xr * cos) + (rot * sin), xp], dim=-1)


def recurrent_gated_delta_rule(q, k, v, g, beta, state):
    """Token-serial gated delta rule.  q,k [S,H,K], v [S,H,V], g,beta [S,H],
    state [H,K,V] f32 or None.  Decay first, then read (prefill.cu:508-522)."""
    dt = q.dtype
    q = l2norm(q)
    k = l2norm(k)
    q, k, v, beta, g = [x.transpose(0, 1).contiguous().to(torch.float32) for x in (q, k, v, beta, g)]
    H, S, K = k.shape
    V = v.shape[-1]
    q = q * (1 / (K ** 0.5))
    out = torch.zeros(H, S, V)
    st = torch.zeros(H, K, V) if state is None else state.to(torch.float32)
    for i in range(S):
        g_t = g[:, i].exp()[:, None, None]
        st = st * g_t
        kv_mem = (st * k[:, i].unsqueeze(-1)).sum(dim=-2)
        delta = (v[:, i] - kv_mem) * beta[:, i].unsqueeze(-1)
        st = st + k[:, i].unsqueeze(-1) * delta.unsqueeze(-2)
        out[:, i] = (st * q[:, i].unsqueeze(-1)).sum(dim=-2)
    return out.transpose(0, 1).contiguous().to(dt), st


def chunk_gated_delta_rule(q, k, v, g, beta, chunk: int = 64, state=None):
    """Chunked (WY) form of the same rule, chunk 64, all f32.  Shapes as above."""
    dt = q.dtype
    q = l2norm(q)
    k = l2norm(k)
    q, k, v, beta, g = [x.transpose(0, 1).contiguous().to(torch.float32) for x in (q, k, v, beta, g)]
    H, S, K = k.shape
    V = v.shape[-1]
    pad = (chunk - S % chunk) % chunk
    q = F.pad(q, (0, 0, 0, pad))
    k = F.pad(k, (0, 0, 0, pad))
    v = F.pad(v, (0, 0, 0, pad))
    beta = F.pad(beta, (0, pad))
    g = F.pad(g, (0, pad))
    T = S + pad
    q = q * (1 / (K ** 0.5))
    v_beta = v * beta.unsqueeze(-1)
    k_beta = k * beta.unsqueeze(-1)
    q, k, v, k_beta, v_beta = [x.reshape(H, -1, chunk, x.shape[-1]) for x in (q, k, v, k_beta, v_beta)]
    g = g.reshape(H, -1, chunk)
    upper = torch.triu(torch.ones(chunk, chunk, dtype=torch.bool), diagonal=0)
    g = g.cumsum(dim=-1)
    decay = ((g.unsqueeze(-1) - g.unsqueeze(-2)).tril().exp().float()).tril()
    attn = -((k_beta @ k.transpose(-1, -2)) * decay).masked_fill(upper, 0)
    for i in range(1, chunk):
        row = attn[..., i, :i].clone()
        sub = attn[..., :i, :i].clone()
        attn[..., i, :i] = row + (row.unsqueeze(-1) * sub).sum(-2)
    attn = attn + torch.eye(chunk, dtype=attn.dtype)
    v = attn @ v_beta
    k_cumdecay = attn @ (k_beta * g.exp().unsqueeze(-1))
    st = torch.zeros(H, K, V) if state is None else state.to(torch.float32)
    out = torch.zeros_like(v)
    strict = torch.triu(torch.ones(chunk, chunk, dtype=torch.bool), diagonal=1)
    for i in range(T // chunk):
        q_i, k_i, v_i = q[:, i], k[:, i], v[:, i]
        a = (q_i @ k_i.transpose(-1, -2) * decay[:, i]).masked_fill_(strict, 0)
        v_prime = k_cumdecay[:, i] @ st
        v_new = v_i - v_prime
        inter = (q_i * g[:, i, :, None].exp()) @ st
        out[:, i] = inter + a @ v_new
        st = (st * g[:, i, -1, None, None].exp()
              + (k_i * (g[:, i, -1, None] - g[:, i]).exp()[..., None]).transpose(-1, -2) @ v_new)
    out = out.reshape(H, -1, V)[:, :S]
    return out.transpose(0, 1).contiguous().to(dt), st


class Oracle:
    """Stateful CPU model: `prefill(ids)` (chunk-64 form, fresh state) then `step(tok)`
    (recurrent form).  State layouts are HuggingFace's: DeltaNet state [layer, head, k, v]
    f32 (the reference stores the transpose [head][v][k], kernel.cu:684), conv state
    [layer, channel, 4] with the newest input last, K/V [layer, kv_head, pos, head_dim]."""

    def __init__(self, weights: dict, dims, max_seq_len: int = 2048, state_dtype=torch.float32):
        """`state_dtype` is the dtype the DeltaNet state is *stored* in between calls.  The
        reference keeps it in f32 (model.py:538, kernel.cu:684-695) and that is the default.
        transformers 5.5.0's cache stores it in the dtype of the conv state (bf16); passing
        torch.bfloat16 reproduces that, so the oracle can be pinned against the unmodified
        library as well."""
        self.w = weights
        self.d = dims
        self.max_seq_len = max_seq_len
        self.state_dtype = state_dtype
        self.keep_all = False        # True: _forward also records every position's hidden state per layer (teacher forcing of prefill)
        self.reset()

    def reset(self):
        d = self.d
        self.position = 0
        self.dn_state = [None] * d.n_dn
        self.conv_state = [None] * d.n_dn
        self.k_cache = [None] * d.n_fa
        self.v_cache = [None] * d.n_fa
        self.last_hidden = None      # [S, hidden] bf16, output of the last layer (pre final norm)
        self.trace = []              # per layer: output hidden of the last position of the last call
        self.trace_all = []          # per layer: output hidden of every position of the last call (only if keep_all)

    # ---- layer bodies -------------------------------------------------------------------
    def _deltanet(self, i_dn: int, p: list, x: torch.Tensor, use_state: bool) -> torch.Tensor:
        d = self.d
        S = x.shape[0]
        mixed = linear(x, p[1]).transpose(0, 1)[None]          # [1, C, S]
        z = linear(x, p[2]).reshape(S, d.dn_heads, d.dn_value_dim)
        b = linear(x, p[3])
        a = linear(x, p[4])
        conv_w = p[5].squeeze(1)                                   # [C, 4]
        kw = d.dn_conv_kernel
        if use_state:
            cs = self.conv_state[i_dn]
            new = torch.cat([cs, mixed], dim=-1).to(conv_w.dtype)
            self.conv_state[i_dn] = new[:, :, -kw:].contiguous()
            out = F.conv1d(new, conv_w.unsqueeze(1), None, padding=0, groups=new.shape[1])
            mixed = F.silu(out[:, :, -S:]).to(x.dtype)
        else:
            self.conv_state[i_dn] = F.pad(mixed, (kw - S, 0)).contiguous()
            mixed = F.silu(F.conv1d(mixed, conv_w.unsqueeze(1), None, padding=kw - 1,
                                    groups=mixed.shape[1])[:, :, :S])
        mixed = mixed[0].transpose(0, 1)                           # [S, C]
        q, k, v = torch.split(mixed, [d.dn_qk_size, d.dn_qk_size, d.dn_v_size], dim=-1)
        q = q.reshape(S, d.dn_k_heads, d.dn_key_dim)
        k = k.reshape(S, d.dn_k_heads, d.dn_key_dim)
        v = v.reshape(S, d.dn_heads, d.dn_value_dim)
        beta = b.sigmoid()
        g = -p[6].float().exp() * F.softplus(a.float() + p[7])
        rep = d.dn_heads // d.dn_k_heads
        if rep > 1:
            q = q.repeat_interleave(rep, dim=1)
            k = k.repeat_interleave(rep, dim=1)
        if use_state:
            o, st = recurrent_gated_delta_rule(q, k, v, g, beta, self.dn_state[i_dn])
        else:
            o, st = chunk_gated_delta_rule(q, k, v, g, beta, 64, None)
        self.dn_state[i_dn] = st.to(self.state_dtype)
        o = gated_rmsnorm(o.reshape(-1, d.dn_value_dim), z.reshape(-1, d.dn_value_dim), p[8], d.rms_eps)
        return linear(o.reshape(S, -1), p[9])

    def _attention(self, i_fa: int, p: list, x: torch.Tensor, cos, sin) -> torch.Tensor:
        d = self.d
        S = x.shape[0]
        hd = d.fa_head_dim
        qg = linear(x, p[1]).view(S, d.fa_q_heads, 2 * hd)
        q, gate = torch.chunk(qg, 2, dim=-1)
        gate = gate.reshape(S, -1)
        q = rmsnorm(q, p[4], d.rms_eps).transpose(0, 1)                      # [Hq, S, hd]
        k = rmsnorm(linear(x, p[2]).view(S, d.fa_kv_heads, hd), p[5], d.rms_eps).transpose(0, 1)
        v = linear(x, p[3]).view(S, d.fa_kv_heads, hd).transpose(0, 1)
        q = apply_rope(q, cos, sin)
        k = apply_rope(k, cos, sin)
        if self.k_cache[i_fa] is not None:
            k = torch.cat([self.k_cache[i_fa], k], dim=1)
            v = torch.cat([self.v_cache[i_fa], v], dim=1)
        self.k_cache[i_fa], self.v_cache[i_fa] = k, v
        rep = d.fa_q_heads // d.fa_kv_heads
        ks = k.repeat_interleave(rep, dim=0)
        vs = v.repeat_interleave(rep, dim=0)
        w = torch.matmul(q, ks.transpose(1, 2)) * (hd ** -0.5)
        L = ks.shape[1]
        if S > 1:
            neg = torch.finfo(w.dtype).min
            qpos = torch.arange(L - S, L)[:, None]
            mask = torch.where(torch.arange(L)[None, :] <= qpos, 0.0, neg).to(w.dtype)
            w = w + mask
        w = F.softmax(w, dim=-1, dtype=torch.float32).to(q.dtype)
        o = torch.matmul(w, vs).transpose(0, 1).contiguous().reshape(S, -1)
        o = o * torch.sigmoid(gate)
        return linear(o, p[6])

    def _forward(self, ids: torch.Tensor, use_state: bool, teacher=None) -> torch.Tensor:
        """teacher: optional per-layer list of [S, hidden] inputs; layer l > 0 then reads teacher[l] instead of the
        previous layer's output (the layer-level comparison the GPU tests make)."""
        d = self.d
        S = ids.numel()
        if self.position + S > self.max_seq_len:
            raise ValueError("sequence exceeds max_seq_len")
        h = F.embedding(ids.long(), self.w["embed_weight"])
        pos = torch.arange(self.position, self.position + S)
        cos, sin = rope_tables(pos, d.fa_rotary_dim, d.rope_theta, h.dtype)
        i_dn = i_fa = 0
        self.trace = []
        self.trace_all = []
        for li, ld in enumerate(self.w["layer_data"]):
            p = ld["ptrs"]
            if teacher is not None and li > 0:
                h = teacher[li].reshape(S, -1)
            x = rmsnorm(h, p[0], d.rms_eps)
            if ld["type"] == 1:
                y = self._attention(i_fa, p, x, cos, sin)
                i_fa += 1
                post, gate_w, up_w, down_w = p[7], p[8], p[9], p[10]
            else:
                y = self._deltanet(i_dn, p, x, use_state)
                i_dn += 1
                post, gate_w, up_w, down_w = p[10], p[11], p[12], p[13]
            h = h + y
            x = rmsnorm(h, post, d.rms_eps)
            h = h + linear(F.silu(linear(x, gate_w)) * linear(x, up_w), down_w)
            self.trace.append(h[-1])
            if self.keep_all:
                self.trace_all.append(h)
        self.position += S
        self.last_hidden = h
        return h

    # ---- public ---------------------------------------------------------------------------
    @torch.no_grad()
    def logits_from_hidden(self, h: torch.Tensor) -> torch.Tensor:
        """Final RMSNorm + tied LM head; bf16 logits (kernel.cu:747-814 takes their arg-max)."""
        return linear(rmsnorm(h, self.w["final_norm_weight"], self.d.rms_eps), self.w["lm_head_weight"])

    @torch.no_grad()
    def prefill(self, ids: torch.Tensor, all_logits: bool = False) -> torch.Tensor:
        """Fresh-state forward over the whole prompt (chunk-64 DeltaNet).  Returns the bf16
        logits of the last position ([V]) or of all positions ([S, V])."""
        self.reset()
        h = self._forward(ids, use_state=False)
        return self.logits_from_hidden(h if all_logits else h[-1])

    @torch.no_grad()
    def step(self, token: int, teacher=None) -> torch.Tensor:
        """One cached decode step (recurrent DeltaNet form).  Returns bf16 logits [V]."""
        use_state = self.position > 0
        h = self._forward(torch.tensor([int(token)]), use_state=use_state, teacher=teacher)
        return self.logits_from_hidden(h[-1])

    @torch.no_grad()
    def generate(self, ids: torch.Tensor, n_new: int):
        """Greedy: prefill, then `n_new` tokens.  torch.argmax on CPU returns the lowest
        index among equal maxima.  Returns (tokens list, list of bf16 logits per step)."""
        logits = self.prefill(ids)
        toks, all_logits = [], []
        for _ in range(n_new):
            all_logits.append(logits)
            t = int(torch.argmax(logits))
            toks.append(t)
            if len(toks) == n_new:
                break
            logits = self.step(t)
        return toks, all_logits

    # ---- state export in the reference's layouts ----------------------------------------
    def dn_states_ref_layout(self) -> torch.Tensor:
        """[n_dn, heads, v, k] f32 -- the value-major layout of kernel.cu:684."""
        return torch.stack([s.transpose(-1, -2).contiguous() for s in self.dn_state])

    def conv_ref_layout(self) -> torch.Tensor:
        """[n_dn, channels, 4] f32 (model.py:539), newest input last."""
        return torch.stack([c[0].float() for c in self.conv_state])
