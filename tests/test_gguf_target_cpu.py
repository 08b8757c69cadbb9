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
    wr.write_header_to_file(); wr.write_kv_data_to_file(); wr.write_tensors_to_file(); wr.close()
    with pytest.raises(TypeError, match="attn_q.weight.*Q8_0"):
        load_gguf_target(path, device="cpu")
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
