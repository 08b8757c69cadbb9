"""TEST INFRASTRUCTURE ONLY: CPU oracle of the tree-verify pass (imported by tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py, never by the product).

Parity status: **parity unpinned** for the forward arithmetic.  The reference builds this pass from ggml operators of
a llama.cpp fork (submodule `deps/llama.cpp`, https://github.com/Luce-Org/llama.cpp.git branch luce-dflash, no commit
recorded, directory empty in the reference checkout), and its own tests store no expected values for it
(models/qwen35_27b/test/smoke_target_forward.cpp:7-8).  What IS pinned: the Q4_K unpacking, against gguf-py 0.19.0
`gguf.quants.dequantize` (tests/test_q4k_oracle.py).  The rest restates the graph semantics of
models/qwen35_27b/src/qwen35_target_graph.cpp:281-804 and the tree semantics of models/qwen35_27b/test/test_dflash.cpp
:396-442, 1355-1521 as "a node's result is the sequential model run on its root-to-node token path", written
path-recursively (no mask, no DFS tricks) so it checks the mask / parent-chain logic of the product independently.

Rounding points (shared with the product by definition, since nothing upstream pins them): activations between
operators are bf16; a Q4_K linear uses the bf16 weight operand of `q4k_gemm_operand` (embedding rows: bf16 of the
published dequantisation) with f32 accumulation and returns bf16; norms, RoPE,
softmax, conv, the delta rule and its state are f32; attention probabilities are rounded to bf16 before P.V; a node's
DeltaNet post-state is kept as f16 and a node that is not its parent's first child (DFS index parent+1) starts from
that f16 copy (qwen35_target_graph.cpp:540-583: the kernel reloads state at DFS branch transitions)."""
import numpy as np
import torch


def q4k_dequant(blocks: np.ndarray) -> np.ndarray:
    """[n, 144] uint8 -> [n, 256] f32: y = (d*sc)*q - (dmin*m), sub-block j of 32 weights uses scale/min j; the low
    nibbles of bytes 32g..32g+31 are weights 64g..64g+31, the high nibbles weights 64g+32..64g+63."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, 144)
    n = blocks.shape[0]
    d = blocks[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(n)
    dmin = blocks[:, 2:4].copy().view(np.float16).astype(np.float32).reshape(n)
    s = blocks[:, 4:16].astype(np.int32)
    sc = np.zeros((n, 8), np.int32); mn = np.zeros((n, 8), np.int32)
    for j in range(8):
        if j < 4:
            sc[:, j] = s[:, j] & 63; mn[:, j] = s[:, j + 4] & 63
        else:
            sc[:, j] = (s[:, j + 4] & 0xF) | ((s[:, j - 4] >> 6) << 4)
            mn[:, j] = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
    qs = blocks[:, 16:144]
    out = np.zeros((n, 256), np.float32)
    for g in range(4):
        q = qs[:, 32 * g:32 * g + 32]
        for half, vals in ((0, q & 0xF), (1, q >> 4)):
            j = 2 * g + half
            dj = (d * sc[:, j].astype(np.float32)).astype(np.float32)[:, None]
            mj = (dmin * mn[:, j].astype(np.float32)).astype(np.float32)[:, None]
            out[:, 64 * g + 32 * half:64 * g + 32 * half + 32] = (dj * vals.astype(np.float32)).astype(np.float32) - mj
    return out


def _f64_to_bf16_once(x: np.ndarray) -> np.ndarray:
    """f64 -> bf16 with ONE round-to-nearest-even (returned as f32): first to f32 with round-to-odd (truncate toward
    zero, set the last bit if anything was lost), which makes the second rounding to 8 bits safe."""
    y = x.astype(np.float32)
    over = np.abs(y.astype(np.float64)) > np.abs(x)
    y = np.where(over, np.nextafter(y, np.float32(0)), y).astype(np.float32)
    inexact = y.astype(np.float64) != x
    bits = y.view(np.uint32)
    y = np.where(inexact, bits | np.uint32(1), bits).astype(np.uint32).view(np.float32)
    return torch.from_numpy(y.copy()).bfloat16().float().numpy()


def q4k_gemm_operand(blocks: np.ndarray) -> np.ndarray:
    """[n, 144] uint8 -> [n, 256] f32 holding the bf16 weight operand of the product's Q4_K GEMM:
    fma_bf16(q, bf16(d*sc), -bf16(dmin*m)) -- d*sc and dmin*m are exact in f32, rounded once to bf16; the fused
    multiply-add is evaluated exactly in f64 and rounded once to bf16."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, 144)
    n = blocks.shape[0]
    d = blocks[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(n)
    dmin = blocks[:, 2:4].copy().view(np.float16).astype(np.float32).reshape(n)
    s = blocks[:, 4:16].astype(np.int32)
    qs = blocks[:, 16:144]
    out = np.zeros((n, 256), np.float32)
    tobf = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).bfloat16().float().numpy().astype(np.float64)   # noqa: E731
    for j in range(8):
        if j < 4:
            sc = s[:, j] & 63; mn = s[:, j + 4] & 63
        else:
            sc = (s[:, j + 4] & 0xF) | ((s[:, j - 4] >> 6) << 4)
            mn = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
        dsc = tobf(d * sc.astype(np.float32))[:, None]
        mm = tobf(dmin * mn.astype(np.float32))[:, None]
        g, half = j // 2, j % 2
        q = qs[:, 32 * g:32 * g + 32]
        q = (q >> 4) if half else (q & 0xF)
        out[:, 32 * j:32 * j + 32] = _f64_to_bf16_once(q.astype(np.float64) * dsc - mm)
    return out


def q8_0_quant(x: np.ndarray) -> np.ndarray:
    """Q8_0 packing of f32 rows [..., 32k] -> uint8 [..., 34k]: per 32 elements f16 d = amax / 127 then 32 int8
    q = round-half-away(x * (1 / d)) with the UNROUNDED f32 d (d = 0 -> all zero), as ggml's quantize_row_q8_0 and
    gguf-py's Q8_0.quantize_blocks do.  Pinned bit for bit to gguf-py 0.19.0 (tests/golden/q8_0_golden.npz)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    blk = x.reshape(-1, 32)
    d = np.abs(blk).max(axis=1, keepdims=True) / np.float32(127)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    y = blk * inv
    q = (np.sign(y) * np.floor(np.abs(y) + np.float32(0.5))).astype(np.int8)        # roundf: halves away from zero
    out = np.empty((blk.shape[0], 34), np.uint8)
    out[:, :2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(*x.shape[:-1], x.shape[-1] // 32 * 34)


def q8_0_dequant(b: np.ndarray) -> np.ndarray:
    """uint8 [..., 34k] -> f32 [..., 32k]: d (f16 -> f32) * q."""
    blk = np.ascontiguousarray(b, dtype=np.uint8).reshape(-1, 34)
    d = blk[:, :2].copy().view(np.float16).astype(np.float32)
    q = blk[:, 2:].copy().view(np.int8).astype(np.float32)
    return (d * q).reshape(*b.shape[:-1], b.shape[-1] // 34 * 32)


def q8_0_cache_value(x: torch.Tensor) -> torch.Tensor:
    """What a Q8_0 cache row written from f32 values x holds: d * q, exact in f32 (11 + 7 significant bits), so that
    quantising it again gives back the same bytes.  The attention reads it as the bf16 operand bf16(d * q): the oracle
    applies that rounding where it uses K and V."""
    return torch.from_numpy(q8_0_dequant(q8_0_quant(x.numpy())))


def q4_0_quant(x: np.ndarray) -> np.ndarray:
    """Q4_0 packing of f32 rows [..., 32k] -> uint8 [..., 18k]: per 32 elements, with m the element of largest magnitude
    (the first one among equals, sign kept): f16 d = m / -8, q = min(15, trunc(x * (1 / d) + 8.5)) with the UNROUNDED f32 d
    (d = 0 -> all q = 8), byte j = q[j] | q[j + 16] << 4, as ggml's quantize_row_q4_0_ref and gguf-py's
    Q4_0.quantize_blocks do.  Pinned bit for bit to gguf-py 0.19.0 (tests/golden/q4_0_golden.npz)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    blk = x.reshape(-1, 32)
    imax = np.abs(blk).argmax(axis=1)[:, None]
    d = np.take_along_axis(blk, imax, axis=1) / np.float32(-8)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    q = np.clip(np.trunc(blk * inv + np.float32(8.5)), 0, 15).astype(np.uint8)
    out = np.empty((blk.shape[0], 18), np.uint8)
    out[:, :2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << np.uint8(4))
    return out.reshape(*x.shape[:-1], x.shape[-1] // 32 * 18)


def q4_0_dequant(b: np.ndarray) -> np.ndarray:
    """uint8 [..., 18k] -> f32 [..., 32k]: d (f16 -> f32) * (q - 8); low nibbles are elements 0..15, high nibbles 16..31."""
    blk = np.ascontiguousarray(b, dtype=np.uint8).reshape(-1, 18)
    d = blk[:, :2].copy().view(np.float16).astype(np.float32)
    qs = blk[:, 2:]
    q = np.concatenate([qs & np.uint8(15), qs >> np.uint8(4)], axis=1).astype(np.float32) - np.float32(8)
    return (d * q).reshape(*b.shape[:-1], b.shape[-1] // 18 * 32)


def kv_cache_value(x: torch.Tensor, kv_type: str) -> torch.Tensor:
    """What a cache row of the given type written from f32 values x holds, as f32 (the attention reads it rounded to bf16)."""
    if kv_type == "q8_0":
        return q8_0_cache_value(x)
    if kv_type == "q4_0":
        return torch.from_numpy(q4_0_dequant(q4_0_quant(x.numpy())))
    if kv_type == "f16":
        return x.half().float()
    raise ValueError(kv_type)


def rb(x: torch.Tensor) -> torch.Tensor:
    return x.bfloat16().float()


class TreeOracle:
    def __init__(self, dims, weights, max_ctx, kv_q8=False, kv_type=None):
        """weights: the dict of qwen35_b200.tree_verify.make_random_tree_weights on the CPU.  kv_type: "bf16", or one of
        the reference's cache types (qwen35_target_graph.cpp:110-122) "q8_0" (its default; kv_q8=True means the same),
        "q4_0", "f16": rows are converted from their f32 values when written and read back rounded to bf16."""
        self.D, self.max_ctx = dims, max_ctx
        self.kv_type = kv_type or ("q8_0" if kv_q8 else "bf16")
        D = dims

        def mat(blocks):
            # numpy releases the interpreter lock inside its array operations, so slices of a large matrix convert in parallel
            r, nb, _ = blocks.shape
            flat = blocks.numpy().reshape(-1, 144)
            if flat.shape[0] < (1 << 16):
                return torch.from_numpy(q4k_gemm_operand(flat)).reshape(r, nb * 256)
            import os
            from concurrent.futures import ThreadPoolExecutor
            nthr = max(1, min(16, os.cpu_count() or 1))
            parts = np.array_split(np.arange(flat.shape[0]), nthr * 4)
            with ThreadPoolExecutor(nthr) as ex:
                outs = list(ex.map(lambda ix: q4k_gemm_operand(flat[ix[0]:ix[-1] + 1]), [p for p in parts if len(p)]))
            return torch.from_numpy(np.concatenate(outs, 0)).reshape(r, nb * 256)

        self.layers = []
        for L in weights["layers"]:
            M = {k: (mat(v) if v.dtype == torch.uint8 else v.float()) for k, v in L.items()}
            self.layers.append(M)
        self.embd_blocks = weights["token_embd"]
        self.output_norm = weights["output_norm"].float()
        self.output_w = mat(weights["output_w"]) if weights["output_w"].dtype == torch.uint8 else weights["output_w"].float()
        # committed context
        self.k = [torch.zeros(D.kv_heads, 0, D.head_dim) for _ in range(D.n_fa)]
        self.v = [torch.zeros(D.kv_heads, 0, D.head_dim) for _ in range(D.n_fa)]
        self.ssm = [torch.zeros(D.dn_v_heads, D.dn_dim, D.dn_dim) for _ in range(D.n_dn)]       # [head][value][key]
        self.conv = [torch.zeros(3, D.conv_ch) for _ in range(D.n_dn)]                           # row 2 newest
        self.past = 0

    # ---- one token through the model, from an explicit context; returns logits and the new context ----
    def _norm(self, x, w):
        return rb(x * torch.rsqrt((x * x).mean() + self.D.rms_eps) * w)

    def _rope(self, x, pos):
        D = self.D
        half = D.rot_dim // 2
        i = torch.arange(half, dtype=torch.float32)
        inv = torch.pow(torch.tensor(D.rope_theta, dtype=torch.float32), -(2 * i) / D.rot_dim)
        ang = (torch.tensor(float(pos), dtype=torch.float32) * inv)
        c, s = torch.cos(ang), torch.sin(ang)
        y = x.clone()
        y[..., :half] = x[..., :half] * c - x[..., half:D.rot_dim] * s
        y[..., half:D.rot_dim] = x[..., half:D.rot_dim] * c + x[..., :half] * s
        return y

    def step(self, token, ctx, pos):
        """ctx = dict(k, v: lists [kv, len, 256] bf16-valued f32; ssm: list f32; conv: list [3, ch]).  Returns
        (logits bf16-valued f32 [vocab], new ctx, per-layer hidden list)."""
        D = self.D
        nb = D.hidden // 256
        if self.embd_blocks.dtype == torch.uint8:
            x = rb(torch.from_numpy(q4k_dequant(self.embd_blocks[token].numpy().reshape(nb, 144))).reshape(D.hidden))
        else:                                   # a dense bf16 table
            x = self.embd_blocks[token].float()
        new = {"k": [], "v": [], "ssm": [], "conv": []}
        hid = []
        i_fa = i_dn = 0
        for il, W in enumerate(self.layers):
            n = self._norm(x, W["attn_norm"])
            proj = rb(W["w_in"] @ n)
            if D.is_fa(il):
                qg = proj[:2 * D.q_heads * 256].reshape(D.q_heads, 2, 256)
                q, gate = qg[:, 0], qg[:, 1]
                kk = proj[2 * D.q_heads * 256:2 * D.q_heads * 256 + D.kv_heads * 256].reshape(D.kv_heads, 256)
                vv = proj[2 * D.q_heads * 256 + D.kv_heads * 256:].reshape(D.kv_heads, 256)
                hn = lambda t, w: t * torch.rsqrt((t * t).mean(-1, keepdim=True) + D.rms_eps) * w      # noqa: E731
                q = rb(self._rope(hn(q, W["q_norm"]), pos))
                kk = self._rope(hn(kk, W["k_norm"]), pos)
                if self.kv_type != "bf16":
                    kk, vv = kv_cache_value(kk, self.kv_type), kv_cache_value(vv, self.kv_type)
                else:
                    kk = rb(kk)
                K = torch.cat([ctx["k"][i_fa], kk[:, None]], 1); V = torch.cat([ctx["v"][i_fa], vv[:, None]], 1)
                new["k"].append(K); new["v"].append(V)
                gqa = D.q_heads // D.kv_heads
                out = torch.zeros(D.q_heads, 256)
                Kb, Vb = rb(K), rb(V)                        # the tensor-core operands (identity for a bf16 cache)
                for h in range(D.q_heads):
                    s = (Kb[h // gqa] @ q[h]) * 0.0625
                    p = torch.exp(s - s.max()); p = rb(p / p.sum())
                    out[h] = p @ Vb[h // gqa]
                att = rb(out * torch.sigmoid(gate)).reshape(-1)
                i_fa += 1
            else:
                xin = proj[:D.conv_ch]; z = proj[D.conv_ch:].reshape(D.dn_v_heads, D.dn_dim)
                ba = rb(W["w_ba"] @ n)
                win = torch.cat([ctx["conv"][i_dn], xin[None]], 0)                                    # [4, ch]
                cw = W["conv_w"]
                s = cw[:, 0] * win[0]
                for t in (1, 2, 3):
                    s = torch.addcmul(s, cw[:, t], win[t])
                c = s * torch.sigmoid(s)
                new["conv"].append(win[1:].clone())
                nk = D.dn_k_heads * D.dn_dim
                q = c[:nk].reshape(D.dn_k_heads, D.dn_dim); k = c[nk:2 * nk].reshape(D.dn_k_heads, D.dn_dim)
                v = c[2 * nk:].reshape(D.dn_v_heads, D.dn_dim)
                q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + D.rms_eps) * 0.08838834764831845
                k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + D.rms_eps)
                beta = torch.sigmoid(ba[:D.dn_v_heads])
                a = ba[D.dn_v_heads:] + W["dt_bias"]
                sp = torch.where(a > 20, a, torch.log1p(torch.exp(a)))
                decay = torch.exp(sp * W["ssm_a"])
                S = ctx["ssm"][i_dn].clone()
                o = torch.zeros(D.dn_v_heads, D.dn_dim)
                for h in range(D.dn_v_heads):
                    kh = h % D.dn_k_heads
                    Sh = S[h] * decay[h]
                    kv = Sh @ k[kh]
                    delta = (v[h] - kv) * beta[h]
                    Sh = Sh + delta[:, None] * k[kh][None, :]
                    o[h] = Sh @ q[kh]
                    S[h] = Sh
                new["ssm"].append(S)
                inv = torch.rsqrt((o * o).mean(-1, keepdim=True) + D.rms_eps)
                att = rb(o * inv * W["ssm_norm"] * (z * torch.sigmoid(z))).reshape(-1)
                i_dn += 1
            r = rb(rb(W["w_out"] @ att) + x)
            n2 = self._norm(r, W["post_norm"])
            g = rb(W["w_gate_up"][:D.ffn] @ n2); u = rb(W["w_gate_up"][D.ffn:] @ n2)
            m = rb(rb(g * torch.sigmoid(g)) * u)
            x = rb(rb(W["w_down"] @ m) + r)
            hid.append(x.clone())
        logits = rb(self.output_w @ self._norm(x, self.output_norm))
        return logits, new, hid

    def context(self):
        return {"k": self.k, "v": self.v, "ssm": self.ssm, "conv": self.conv}

    def feed(self, tokens):
        """Sequentially extend the committed context (f32 state, no f16 rounding)."""
        for t in tokens:
            _, ctx, _ = self.step(int(t), self.context(), self.past)
            self.k, self.v, self.ssm, self.conv = ctx["k"], ctx["v"], ctx["ssm"], ctx["conv"]
            self.past += 1

    def verify(self, tokens, parents):
        """Per-node logits, per-node contexts (post-state as the product persists it) and hidden traces."""
        n = len(tokens)
        children = [[] for _ in range(n)]
        for t in range(1, n):
            children[parents[t]].append(t)
        logits, ctxs, hids, depth = [None] * n, [None] * n, [None] * n, [0] * n

        def run(t, ctx_in):
            logits[t], c, hids[t] = self.step(int(tokens[t]), ctx_in, self.past + depth[t])
            ctxs[t] = c
            for ch in children[t]:
                depth[ch] = depth[t] + 1
                if ch == t + 1:
                    cin = c
                else:                      # DFS branch transition: the child starts from the persisted f16 state
                    cin = dict(c); cin["ssm"] = [s.half().float() for s in c["ssm"]]
                run(ch, cin)

        run(0, self.context())
        return logits, ctxs, hids

    @staticmethod
    def accept(tokens, parents, argmax):
        path, cur = [0], 0
        while True:
            nxt = [c for c in range(cur + 1, len(tokens)) if parents[c] == cur and int(tokens[c]) == int(argmax[cur])]
            if not nxt:
                break
            cur = nxt[0]; path.append(cur)
        return path, int(argmax[cur])

    def commit(self, ctxs, path):
        leaf = ctxs[path[-1]]
        self.k, self.v, self.conv = leaf["k"], leaf["v"], leaf["conv"]
        self.ssm = [s.half().float() for s in leaf["ssm"]]
        self.past += len(path)
