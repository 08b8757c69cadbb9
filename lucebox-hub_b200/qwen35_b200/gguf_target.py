"""GGUF ingestion for the tree-verify target: the role of the reference's models/qwen35_27b/src/gguf_target_loader.cpp
(tensor names :7-39, hyper-parameter keys :218-232).  Reads the file with gguf-py's reader (memory mapped), checks the
`qwen35` hyper-parameters, and assembles the weight layout of `Qwen35TreeLayer`: matrices that the pass consumes fused
(q|k|v, qkv|z, gate|up) are row concatenations of the tensors' raw super-block bytes, so nothing is re-quantised.

Matrices whose tensors are all Q4_K stay quantised (the GEMM dequantises in the kernel).  A (fused) matrix with a tensor
of another type -- published mixed files carry Q5_K, Q6_K, Q8_0 and IQ4_XS tensors -- is dequantised on the host with
gguf-py's reference routines and handed over as plain bf16 (`allow_dense=True`, the default; 3.5 x the bytes of Q4_K
for that matrix), or refused by name and type (`allow_dense=False`).  Vectors and the small beta / alpha projections
are F32 / F16 / BF16."""
import numpy as np
import torch

from .tree_verify import TreeDims

ARCH = "qwen35"


def _field(reader, key, default=None):
    f = reader.fields.get(key)
    if f is None:
        if default is None:
            raise KeyError(f"missing gguf key: {key}")
        return default
    v = f.parts[f.data[0]]
    return v.tolist()[0] if v.size == 1 else v.tolist()


def read_dims(reader) -> TreeDims:
    arch = bytes(reader.fields["general.architecture"].parts[reader.fields["general.architecture"].data[0]]).decode()
    if arch != ARCH:
        raise ValueError(f"general.architecture is {arch!r}, expected {ARCH!r}")
    k = lambda s, d=None: _field(reader, f"{ARCH}.{s}", d)      # noqa: E731
    head_dim = int(k("attention.key_length"))
    if int(k("attention.value_length")) != head_dim:
        raise ValueError("key_length and value_length differ")
    if int(k("ssm.conv_kernel")) != 4:
        raise ValueError("ssm.conv_kernel must be 4")
    return TreeDims(n_layers=int(k("block_count")), hidden=int(k("embedding_length")), ffn=int(k("feed_forward_length")), vocab=0,
                    q_heads=int(k("attention.head_count")), kv_heads=int(k("attention.head_count_kv")),
                    dn_k_heads=int(k("ssm.group_count")), dn_v_heads=int(k("ssm.time_step_rank")), head_dim=head_dim,
                    dn_dim=int(k("ssm.state_size")), rot_dim=int(k("rope.dimension_count", 64)), fa_period=int(k("full_attention_interval")),
                    rope_theta=float(k("rope.freq_base", 1.0e7)), rms_eps=float(k("attention.layer_norm_rms_epsilon", 1.0e-6)))


def load_gguf_target(path: str, device="cuda", allow_dense: bool = True):
    """Returns (TreeDims, weights dict for qwen35_b200.tree_verify.TreeTarget)."""
    import dataclasses

    from gguf import GGMLQuantizationType as T
    from gguf import GGUFReader

    reader = GGUFReader(path)
    dims = read_dims(reader)
    tensors = {t.name: t for t in reader.tensors}

    def need(name):
        if name not in tensors:
            raise KeyError(f"tensor {name} missing from {path}")
        return tensors[name]

    def q4k_blocks(t, rows, cols):
        return torch.from_numpy(np.array(t.data, dtype=np.uint8).reshape(rows, cols // 256, 144))

    def dense(t, rows, cols):
        from gguf.quants import dequantize
        if t.tensor_type == T.F32:
            a = np.array(t.data, dtype=np.float32)
        elif t.tensor_type == T.F16:
            a = np.array(t.data, dtype=np.float16).astype(np.float32)
        elif t.tensor_type == T.BF16:
            return torch.from_numpy(np.ascontiguousarray(t.data).view(np.int16).copy()).view(torch.bfloat16).reshape(rows, cols)
        else:
            a = dequantize(np.array(t.data), t.tensor_type).astype(np.float32)
        return torch.from_numpy(a.reshape(rows, cols)).bfloat16()

    def matrix(parts, cols):
        """parts = [(tensor name, rows)]: the row-wise fusion of those tensors, Q4_K blocks if every part is Q4_K."""
        ts = []
        for name, rows in parts:
            t = need(name)
            if [int(x) for x in t.shape] != [cols, rows]:
                raise ValueError(f"{name}: shape {list(t.shape)}, expected [{cols}, {rows}]")
            ts.append((t, rows))
        if all(t.tensor_type == T.Q4_K for t, _ in ts) and cols % 256 == 0:
            return torch.cat([q4k_blocks(t, rows, cols) for t, rows in ts], 0)
        if not allow_dense:
            bad = next(t for t, _ in ts if t.tensor_type != T.Q4_K)
            raise TypeError(f"{bad.name}: type {bad.tensor_type.name} is not supported for a weight matrix (Q4_K only)")
        return torch.cat([dense(t, rows, cols) for t, rows in ts], 0)

    def vec(name, shape):
        t = need(name)
        if t.tensor_type == T.F32:
            a = torch.from_numpy(np.array(t.data, dtype=np.float32))
        elif t.tensor_type == T.F16:
            a = torch.from_numpy(np.array(t.data, dtype=np.float16)).float()
        elif t.tensor_type == T.BF16:
            a = torch.from_numpy(np.ascontiguousarray(t.data).view(np.int16).copy()).view(torch.bfloat16).float()
        else:
            raise TypeError(f"{name}: type {t.tensor_type.name} is not supported for a vector / small matrix")
        return a.reshape(shape).contiguous()

    D = dims
    H = D.hidden
    emb = need("token_embd.weight")
    vocab = int(emb.shape[1])
    D = dataclasses.replace(D, vocab=vocab)
    layers = []
    for il in range(D.n_layers):
        p = f"blk.{il}."
        L = {"attn_norm": vec(p + "attn_norm.weight", (H,)), "post_norm": vec(p + "post_attention_norm.weight", (H,)),
             "w_gate_up": matrix([(p + "ffn_gate.weight", D.ffn), (p + "ffn_up.weight", D.ffn)], H),
             "w_down": matrix([(p + "ffn_down.weight", H)], D.ffn)}
        if D.is_fa(il):
            qd, kvd = D.q_heads * D.head_dim, D.kv_heads * D.head_dim
            L["w_in"] = matrix([(p + "attn_q.weight", 2 * qd), (p + "attn_k.weight", kvd), (p + "attn_v.weight", kvd)], H)
            L["w_out"] = matrix([(p + "attn_output.weight", H)], qd)
            L["q_norm"] = vec(p + "attn_q_norm.weight", (D.head_dim,))
            L["k_norm"] = vec(p + "attn_k_norm.weight", (D.head_dim,))
        else:
            inner = D.dn_v_heads * D.dn_dim
            L["w_in"] = matrix([(p + "attn_qkv.weight", D.conv_ch), (p + "attn_gate.weight", inner)], H)
            L["w_out"] = matrix([(p + "ssm_out.weight", H)], inner)
            L["w_ba"] = torch.cat([vec(p + "ssm_beta.weight", (D.dn_v_heads, H)), vec(p + "ssm_alpha.weight", (D.dn_v_heads, H))], 0).bfloat16()
            L["conv_w"] = vec(p + "ssm_conv1d.weight", (D.conv_ch, 4))
            L["ssm_a"] = vec(p + "ssm_a", (D.dn_v_heads,))
            L["dt_bias"] = vec(p + "ssm_dt.bias", (D.dn_v_heads,))
            L["ssm_norm"] = vec(p + "ssm_norm.weight", (D.dn_dim,))
        layers.append({k: v.to(device) for k, v in L.items()})
    w = {"layers": layers, "token_embd": matrix([("token_embd.weight", vocab)], H).to(device),
         "output_norm": vec("output_norm.weight", (H,)).to(device),
         "output_w": matrix([("output.weight" if "output.weight" in tensors else "token_embd.weight", vocab)], H).to(device)}
    return D, w


def write_gguf_target(path: str, dims: TreeDims, weights: dict):
    """Write a weights dict (as made by make_random_tree_weights) under the reference's tensor names: the inverse of
    load_gguf_target, used to make test files; fused matrices are split back into their tensors."""
    from gguf import GGMLQuantizationType as T
    from gguf import GGUFWriter

    D = dims
    wr = GGUFWriter(path, ARCH)
    k = lambda s: f"{ARCH}.{s}"      # noqa: E731
    wr.add_uint32(k("block_count"), D.n_layers); wr.add_uint32(k("embedding_length"), D.hidden); wr.add_uint32(k("feed_forward_length"), D.ffn)
    wr.add_uint32(k("attention.head_count"), D.q_heads); wr.add_uint32(k("attention.head_count_kv"), D.kv_heads)
    wr.add_uint32(k("attention.key_length"), D.head_dim); wr.add_uint32(k("attention.value_length"), D.head_dim)
    wr.add_uint32(k("full_attention_interval"), D.fa_period); wr.add_uint32(k("ssm.conv_kernel"), 4)
    wr.add_uint32(k("ssm.inner_size"), D.dn_v_heads * D.dn_dim); wr.add_uint32(k("ssm.state_size"), D.dn_dim)
    wr.add_uint32(k("ssm.time_step_rank"), D.dn_v_heads); wr.add_uint32(k("ssm.group_count"), D.dn_k_heads)
    wr.add_uint32(k("rope.dimension_count"), D.rot_dim); wr.add_float32(k("rope.freq_base"), D.rope_theta)
    wr.add_float32(k("attention.layer_norm_rms_epsilon"), D.rms_eps)

    def q(name, blocks):                     # [rows, K/256, 144] uint8
        a = blocks.cpu().numpy()
        wr.add_tensor(name, a.reshape(a.shape[0], -1), raw_dtype=T.Q4_K)

    def f(name, t):
        wr.add_tensor(name, t.float().cpu().numpy())

    q("token_embd.weight", weights["token_embd"]); f("output_norm.weight", weights["output_norm"]); q("output.weight", weights["output_w"])
    for il, L in enumerate(weights["layers"]):
        p = f"blk.{il}."
        f(p + "attn_norm.weight", L["attn_norm"]); f(p + "post_attention_norm.weight", L["post_norm"])
        q(p + "ffn_gate.weight", L["w_gate_up"][:D.ffn]); q(p + "ffn_up.weight", L["w_gate_up"][D.ffn:]); q(p + "ffn_down.weight", L["w_down"])
        if D.is_fa(il):
            qd, kvd = 2 * D.q_heads * D.head_dim, D.kv_heads * D.head_dim
            q(p + "attn_q.weight", L["w_in"][:qd]); q(p + "attn_k.weight", L["w_in"][qd:qd + kvd]); q(p + "attn_v.weight", L["w_in"][qd + kvd:])
            q(p + "attn_output.weight", L["w_out"]); f(p + "attn_q_norm.weight", L["q_norm"]); f(p + "attn_k_norm.weight", L["k_norm"])
        else:
            q(p + "attn_qkv.weight", L["w_in"][:D.conv_ch]); q(p + "attn_gate.weight", L["w_in"][D.conv_ch:]); q(p + "ssm_out.weight", L["w_out"])
            f(p + "ssm_beta.weight", L["w_ba"][:D.dn_v_heads]); f(p + "ssm_alpha.weight", L["w_ba"][D.dn_v_heads:])
            f(p + "ssm_conv1d.weight", L["conv_w"]); f(p + "ssm_a", L["ssm_a"]); f(p + "ssm_dt.bias", L["dt_bias"]); f(p + "ssm_norm.weight", L["ssm_norm"])
    wr.write_header_to_file(); wr.write_kv_data_to_file(); wr.write_tensors_to_file(); wr.close()
