"""CPU: GGUF ingestion of the tree-verify target.  A file written under the reference's tensor names and `qwen35.*`
keys loads back into the same weights (fused matrices re-assembled byte for byte); foreign types are refused."""
import numpy as np
import pytest
import torch

gguf = pytest.importorskip("gguf")


def _small():
    from qwen35_b200.tree_verify import TreeDims, make_random_tree_weights
    D = TreeDims(n_layers=4, hidden=256, ffn=512, vocab=320, q_heads=2, kv_heads=1, dn_k_heads=1, dn_v_heads=2)
    return D, make_random_tree_weights(D, 3)


def test_gguf_round_trip(tmp_path):
    from qwen35_b200.gguf_target import load_gguf_target, write_gguf_target
    D, w = _small()
    path = str(tmp_path / "target.gguf")
    write_gguf_target(path, D, w)
    D2, w2 = load_gguf_target(path, device="cpu")
    import dataclasses
    assert abs(D2.rms_eps - D.rms_eps) < 1e-12 and D2.rope_theta == D.rope_theta          # eps travels as f32
    assert dataclasses.replace(D2, rms_eps=D.rms_eps) == D
    for k in ("token_embd", "output_norm", "output_w"):
        assert torch.equal(w2[k], w[k])
    for a, b in zip(w2["layers"], w["layers"]):
        assert set(a) == set(b)
        for k in a:
            assert a[k].dtype == b[k].dtype and a[k].shape == b[k].shape and torch.equal(a[k], b[k]), k


def test_gguf_refuses_other_quant_types_and_bad_shapes(tmp_path):
    from gguf import GGMLQuantizationType as T
    from gguf import GGUFWriter
    from qwen35_b200.gguf_target import ARCH, load_gguf_target, write_gguf_target
    D, w = _small()
    # a Q8_0 attention matrix (as in published mixed files) is named in the error
    path = str(tmp_path / "mixed.gguf")
    wr = GGUFWriter(path, ARCH)
    for key, v in (("block_count", 1), ("embedding_length", 256), ("feed_forward_length", 512), ("attention.head_count", 2),
                   ("attention.head_count_kv", 1), ("attention.key_length", 256), ("attention.value_length", 256),
                   ("full_attention_interval", 1), ("ssm.conv_kernel", 4), ("ssm.state_size", 128), ("ssm.time_step_rank", 2), ("ssm.group_count", 1)):
        wr.add_uint32(f"{ARCH}.{key}", v)
    wr.add_tensor("token_embd.weight", w["token_embd"].numpy().reshape(320, -1), raw_dtype=T.Q4_K)
    wr.add_tensor("output_norm.weight", np.ones(256, np.float32))
    wr.add_tensor("blk.0.attn_norm.weight", np.ones(256, np.float32)); wr.add_tensor("blk.0.post_attention_norm.weight", np.ones(256, np.float32))
    blk = w["layers"][0]
    wr.add_tensor("blk.0.ffn_gate.weight", blk["w_gate_up"][:512].numpy().reshape(512, -1), raw_dtype=T.Q4_K)
    wr.add_tensor("blk.0.ffn_up.weight", blk["w_gate_up"][512:].numpy().reshape(512, -1), raw_dtype=T.Q4_K)
    wr.add_tensor("blk.0.ffn_down.weight", blk["w_down"].numpy().reshape(256, -1), raw_dtype=T.Q4_K)
    wr.add_tensor("blk.0.attn_q.weight", np.zeros((1024, 256 // 32 * 34), np.uint8), raw_dtype=T.Q8_0)
    wr.add_tensor("blk.0.attn_k.weight", np.zeros((256, 256 // 32 * 34), np.uint8), raw_dtype=T.Q8_0)
    wr.add_tensor("blk.0.attn_v.weight", np.zeros((256, 256 // 32 * 34), np.uint8), raw_dtype=T.Q8_0)
    wr.write_header_to_file(); wr.write_kv_data_to_file(); wr.write_tensors_to_file(); wr.close()
    with pytest.raises(TypeError, match="attn_q.weight.*Q8_0"):
        load_gguf_target(path, device="cpu", allow_dense=False)
    # wrong architecture string
    path2 = str(tmp_path / "arch.gguf")
    wr = GGUFWriter(path2, "llama"); wr.add_uint32("llama.block_count", 1)
    wr.add_tensor("x", np.zeros(4, np.float32)); wr.write_header_to_file(); wr.write_kv_data_to_file(); wr.write_tensors_to_file(); wr.close()
    with pytest.raises(ValueError):
        load_gguf_target(path2, device="cpu")
    # a missing tensor
    path3 = str(tmp_path / "ok.gguf")
    write_gguf_target(path3, D, {**w, "layers": w["layers"]})
    D3, w3 = load_gguf_target(path3, device="cpu")
    assert D3.vocab == 320 and len(w3["layers"]) == 4


def test_gguf_mixed_types_become_dense_bf16(tmp_path):
    """Published files mix quantisation types: a Q8_0 / F16 matrix is dequantised with gguf-py's own routine and handed
    over as bf16; all-Q4_K matrices stay quantised."""
    from gguf import GGMLQuantizationType as T
    from gguf import GGUFWriter
    from gguf.quants import dequantize, quantize
    from qwen35_b200.gguf_target import ARCH, load_gguf_target, write_gguf_target
    D, w = _small()
    base = str(tmp_path / "base.gguf")
    write_gguf_target(base, D, w)
    # rewrite the file with attn_k / attn_v of the attention layer as Q8_0 and the LM head as F16
    from gguf import GGUFReader
    rd = GGUFReader(base)
    rng = np.random.default_rng(0)
    kv = (rng.standard_normal((256, 256)) * 0.05).astype(np.float32)
    q8 = quantize(kv, T.Q8_0)
    head = (rng.standard_normal((D.vocab, 256)) * 0.05).astype(np.float16)
    path = str(tmp_path / "mixed.gguf")
    wr = GGUFWriter(path, ARCH)
    for f in rd.fields.values():
        if f.name.startswith(ARCH + "."):
            v = f.parts[f.data[0]]
            (wr.add_float32 if v.dtype.kind == "f" else wr.add_uint32)(f.name, v.tolist()[0])
    for t in rd.tensors:
        if t.name in ("blk.3.attn_k.weight", "blk.3.attn_v.weight"):
            wr.add_tensor(t.name, q8, raw_dtype=T.Q8_0)
        elif t.name == "output.weight":
            wr.add_tensor(t.name, head)
        else:
            wr.add_tensor(t.name, np.array(t.data), raw_dtype=t.tensor_type if t.tensor_type == T.Q4_K else None)
    wr.write_header_to_file(); wr.write_kv_data_to_file(); wr.write_tensors_to_file(); wr.close()
    D2, w2 = load_gguf_target(path, device="cpu")
    L = w2["layers"][3]
    assert L["w_in"].dtype == torch.bfloat16 and L["w_in"].shape == (D.fa_in, D.hidden)          # fused q|k|v went dense as a whole
    ref_kv = torch.from_numpy(dequantize(q8, T.Q8_0).astype(np.float32)).bfloat16()
    qd = 2 * D.q_heads * D.head_dim
    assert torch.equal(L["w_in"][qd:qd + 256], ref_kv) and torch.equal(L["w_in"][qd + 256:], ref_kv)
    from oracle.tree_verify_oracle import q4k_dequant
    ref_q = torch.from_numpy(q4k_dequant(w["layers"][3]["w_in"][:qd].numpy().reshape(-1, 144))).reshape(qd, D.hidden).bfloat16()
    assert torch.equal(L["w_in"][:qd], ref_q)
    assert w2["output_w"].dtype == torch.bfloat16 and torch.equal(w2["output_w"], torch.from_numpy(head.astype(np.float32)).bfloat16())
    assert w2["layers"][0]["w_in"].dtype == torch.uint8 and w2["token_embd"].dtype == torch.uint8      # untouched matrices stay Q4_K
