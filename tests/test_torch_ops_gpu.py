"""The reference's torch-op boundary: `import qwen35_megakernel_bf16_C` registers the nine ops of
models/qwen35_0p8b/torch_bindings.cpp:529-627; calling them with the reference's argument lists must give what
the Decoder API gives."""
import pytest
import torch

OPS = ["decode", "decode_nvfp4", "decode_many_nvfp4", "prefill_bf16", "prefill_bf16_nvfp4_lm", "prefill_megakernel_nvfp4",
       "prefill_bf16_mega", "quantize_nvfp4_out", "quantize_nvfp4_lm_out"]


def test_ops_are_registered_with_reference_schemas():
    import qwen35_megakernel_bf16_C  # noqa: F401
    ops = torch.ops.qwen35_megakernel_bf16_C
    for name in OPS:
        assert hasattr(ops, name)
    sch = ops.decode.default._schema
    assert [a.name for a in sch.arguments][:6] == ["output_token", "input_token_id", "embed_weight", "layer_weights_packed",
                                                   "final_norm_weight", "lm_head_weight"]
    assert len(sch.arguments) == 28 and [a.name for a in sch.arguments][-2:] == ["position", "max_seq_len"]
    assert len(ops.prefill_bf16.default._schema.arguments) == 28
    assert len(ops.decode_nvfp4.default._schema.arguments) == 34
    assert len(ops.prefill_bf16_nvfp4_lm.default._schema.arguments) == 34


@pytest.mark.gpu
def test_ops_match_decoder_api(full_weights_cpu):
    import qwen35_megakernel_bf16_C  # noqa: F401
    from qwen35_b200.config import QWEN35_0P8B as D
    from qwen35_b200.model import Decoder
    from qwen35_b200.weights import make_token_ids, weights_to
    ops = torch.ops.qwen35_megakernel_bf16_C
    wg = weights_to(full_weights_cpu, "cuda")
    dec = Decoder(weights=wg, backend="nvfp4", max_seq_len=2048)      # holds both the bf16 and the NVFP4 tables
    ids = make_token_ids(40, 9, D.vocab).cuda()
    dummy = torch.zeros(16, device="cuda")
    scratch = [dummy] * 10 + [dummy] * 5

    # ---- bf16: prefill_bf16 then decode, against Decoder (bf16 path called directly) ----
    bdec = Decoder(weights=wg, backend="bf16", max_seq_len=2048)
    first = bdec.prefill_tokens(ids)
    ref = [first] + bdec.step_many(first, 5).tolist()
    bdec.reset()
    b = bdec._ensure_prefill_buffers(40)
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.prefill_bf16(out, ids, bdec._embed_weight, bdec._layer_weights_packed, bdec._prefill_fused_weights_packed,
                     bdec._final_norm_weight, bdec._lm_head_weight, bdec._fa_k_cache, bdec._fa_v_cache, bdec._dn_states, bdec._conv_bufs,
                     b["hidden"], b["residual"], b["normalized"], b["proj_buf"], b["proj_buf2"], dummy, dummy, dummy,
                     b["attn_buf"], b["mlp_buf"], b["dn_out_buf"], b["beta_buf"], b["alpha_buf"], b["final_normed"], b["hidden_bf16_out"],
                     b["lm_bmv"], b["lm_bmi"])
    got = [int(out.item())]
    for i in range(5):
        ops.decode(out, got[-1], bdec._embed_weight, bdec._layer_weights_packed, bdec._final_norm_weight, bdec._lm_head_weight,
                   bdec._fa_k_cache, bdec._fa_v_cache, bdec._dn_states, bdec._conv_bufs, bdec._hidden, *scratch, 40 + i, 2048)
        got.append(int(out.item()))
    assert got == ref

    # ---- single-dispatch bf16 prompt pass: the batched pass without the fused-weight table; agrees with the fused op ----
    t_fused = bdec.prefill_tokens(ids, mode="batched")
    st_fused = bdec._dn_states.clone()
    t_mega = bdec.prefill_tokens(ids, mode="mega")
    st_mega = bdec._dn_states.clone()
    bdec.reset()
    ops.prefill_bf16_mega(out, ids, bdec._embed_weight, bdec._layer_weights_packed, bdec._final_norm_weight, bdec._lm_head_weight,
                          bdec._fa_k_cache, bdec._fa_v_cache, bdec._dn_states, bdec._conv_bufs, b["hidden"], b["residual"], b["normalized"],
                          b["proj_buf"], b["proj_buf2"], b["attn_buf"], b["mlp_buf"], b["dn_out_buf"], b["beta_buf"], b["alpha_buf"],
                          b["final_normed"], b["hidden_bf16_out"], b["lm_bmv"], b["lm_bmi"])
    assert int(out.item()) == t_mega and torch.equal(bdec._dn_states, st_mega)
    assert float((st_mega[0] - st_fused[0]).norm() / st_fused[0].norm()) <= 1e-3 and 0 <= t_fused < D.vocab
    # the C symbol of the same name with the reference's argument list (torch_bindings.cpp:354-364; cache length 2048)
    import ctypes as C
    from qwen35_b200 import _capi
    bdec.reset()
    ptr = lambda t: t.data_ptr()       # noqa: E731
    st = _capi.lib().launch_prefill_bf16_mega(
        ptr(ids), 40, ptr(out), ptr(bdec._embed_weight), ptr(bdec._layer_weights_packed), ptr(bdec._final_norm_weight), ptr(bdec._lm_head_weight),
        ptr(bdec._fa_k_cache), ptr(bdec._fa_v_cache), ptr(bdec._dn_states), ptr(bdec._conv_bufs), ptr(b["hidden"]), ptr(b["residual"]),
        ptr(b["normalized"]), ptr(b["proj_buf"]), ptr(b["proj_buf2"]), ptr(b["attn_buf"]), ptr(b["mlp_buf"]), ptr(b["dn_out_buf"]),
        ptr(b["beta_buf"]), ptr(b["alpha_buf"]), ptr(b["final_normed"]), ptr(b["hidden_bf16_out"]), ptr(b["lm_bmv"]), ptr(b["lm_bmi"]),
        C.c_void_p(torch.cuda.current_stream().cuda_stream))
    _capi.check(st, "launch_prefill_bf16_mega")
    assert int(out.item()) == t_mega and torch.equal(bdec._dn_states, st_mega)

    # ---- NVFP4: token-serial prompt pass, decode_nvfp4, decode_many_nvfp4 ----
    nv_head = [dec._embed_weight, dec._layer_weights_packed_nvfp4, dec._final_norm_weight, dec._lm_head_weight_packed, dec._lm_head_scales,
               dummy, dummy, dummy, dummy]
    nv_state = [dec._fa_k_cache, dec._fa_v_cache, dec._dn_states, dec._conv_bufs, dec._hidden]
    first = dec.prefill_tokens(ids, mode="serial")
    ref = [first] + dec.step_many(first, 6).tolist()
    dec.reset()
    ops.prefill_megakernel_nvfp4(out, ids, *nv_head, *nv_state, *scratch, 2048, 32)
    got = [int(out.item())]
    ops.decode_nvfp4(out, got[-1], *nv_head, *nv_state, *scratch, 40, 2048, 32)
    got.append(int(out.item()))
    many = torch.zeros(5, dtype=torch.int32, device="cuda")
    tokbuf = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.decode_many_nvfp4(many, tokbuf, got[-1], *nv_head, *nv_state, *scratch, 41, 2048, 32)
    got += many.tolist()
    assert got == ref and int(tokbuf.item()) == ref[-1]

    # ---- hybrid prefill: bf16 body, NVFP4 LM head ----
    dec.reset()
    ops.prefill_bf16_nvfp4_lm(out, ids, dec._embed_weight, dec._layer_weights_packed, dec._prefill_fused_weights_packed,
                              dec._final_norm_weight, dec._lm_head_weight, dec._lm_head_weight_packed, dec._lm_head_scales,
                              dec._fa_k_cache, dec._fa_v_cache, dec._dn_states, dec._conv_bufs,
                              b["hidden"], b["residual"], b["normalized"], b["proj_buf"], b["proj_buf2"], dummy, dummy, dummy,
                              b["attn_buf"], b["mlp_buf"], b["dn_out_buf"], b["beta_buf"], b["alpha_buf"], b["final_normed"],
                              b["hidden_bf16_out"], b["lm_bmv"], b["lm_bmi"], dummy, dummy, dummy, dummy)
    assert 0 <= int(out.item()) < D.vocab
    assert torch.equal(dec._dn_states, bdec_state_after_prefill(bdec, ids))

    # ---- packers ----
    w = (torch.randn(256, 1024, device="cuda") * 0.02).bfloat16()
    p1 = torch.empty(256, 512, dtype=torch.uint8, device="cuda"); s1 = torch.empty(256, 32, dtype=torch.float16, device="cuda")
    ops.quantize_nvfp4_out(p1, s1, w, 32)
    from qwen35_b200.model import _quantize_matrix_nvfp4, _quantize_matrix_nvfp4_lm
    q = _quantize_matrix_nvfp4(w, 32)
    assert torch.equal(p1, q["packed"]) and torch.equal(s1, q["scales"])
    p2 = torch.empty(256, 512, dtype=torch.uint8, device="cuda"); s2 = torch.zeros(2 * 16 * 512, dtype=torch.uint8, device="cuda")
    ops.quantize_nvfp4_lm_out(p2, s2, w)
    q = _quantize_matrix_nvfp4_lm(w)
    assert torch.equal(p2, q["packed"]) and torch.equal(s2, q["scales"])
    dec.check_status()


def bdec_state_after_prefill(bdec, ids):
    bdec.prefill_tokens(ids)
    return bdec._dn_states
