"""`import qwen35_megakernel_bf16_C` -- the reference's torch-extension module name.

Importing it registers `torch.ops.qwen35_megakernel_bf16_C.{decode, decode_nvfp4, decode_many_nvfp4,
prefill_bf16, prefill_bf16_nvfp4_lm, prefill_megakernel_nvfp4, prefill_bf16_mega, quantize_nvfp4_out,
quantize_nvfp4_lm_out}` with the schemas of the reference's TORCH_LIBRARY block
(models/qwen35_0p8b/torch_bindings.cpp:529-627), for the CUDA dispatch key only.  Each op unwraps
`data_ptr()`, takes the current CUDA stream and calls the function of libqwen35_b200.so that replaces the
reference launcher; a non-zero status raises.  The reference's unmodified `model.py` can therefore run on top
of this module.  Differences: `max_seq_len` is honoured, scratch tensors are ignored, the prefill ops read
the cache length from `fa_k_cache.size(2)`.
"""
import ctypes as C

import torch

from qwen35_b200 import _capi

_NS = "qwen35_megakernel_bf16_C"
_lib = torch.library.Library(_NS, "DEF")

_DECODE_TAIL = ("Tensor fa_k_cache, Tensor fa_v_cache, Tensor dn_states, Tensor conv_bufs, "
                "Tensor hidden_buffer, Tensor activations, Tensor residual, "
                "Tensor qkv_scratch, Tensor kv_scratch, Tensor attn_out, "
                "Tensor mlp_inter, Tensor z_scratch, Tensor beta_scratch, "
                "Tensor alpha_scratch, Tensor normalized, "
                "Tensor barrier_counter, Tensor barrier_generation, "
                "Tensor block_max_vals, Tensor block_max_idxs, Tensor lm_sync_counter, ")
_NVFP4_HEAD = ("Tensor embed_weight, Tensor layer_weights_packed, "
               "Tensor final_norm_weight, Tensor lm_head_weight_packed, Tensor lm_head_scales, "
               "Tensor lm_hidden_bf16, Tensor lm_hidden_packed, Tensor lm_hidden_scales, Tensor lm_logits_f16, ")
_PREFILL_BUFS = ("Tensor fa_k_cache, Tensor fa_v_cache, Tensor dn_states, Tensor conv_bufs, "
                 "Tensor hidden, Tensor residual, Tensor normalized, ")

_lib.define("decode(Tensor output_token, int input_token_id, Tensor embed_weight, Tensor layer_weights_packed, "
            "Tensor final_norm_weight, Tensor lm_head_weight, " + _DECODE_TAIL + "int position, int max_seq_len) -> ()")
_lib.define("decode_nvfp4(Tensor output_token, int input_token_id, " + _NVFP4_HEAD + _DECODE_TAIL +
            "int position, int max_seq_len, int group_size) -> ()")
_lib.define("decode_many_nvfp4(Tensor output_tokens, Tensor token_buffer, int input_token_id, " + _NVFP4_HEAD + _DECODE_TAIL +
            "int position, int max_seq_len, int group_size) -> ()")
_lib.define("prefill_bf16(Tensor output_token, Tensor token_ids, Tensor embed_weight, Tensor layer_weights_packed, "
            "Tensor prefill_fused_weights_packed, Tensor final_norm_weight, Tensor lm_head_weight, " + _PREFILL_BUFS +
            "Tensor proj_buf, Tensor proj_buf2, Tensor proj_buf_half, Tensor proj_act_packed, Tensor proj_act_scales, "
            "Tensor attn_buf, Tensor mlp_buf, Tensor dn_out_buf, Tensor beta_buf, Tensor alpha_buf, "
            "Tensor final_normed, Tensor hidden_bf16_out, Tensor lm_bmv, Tensor lm_bmi) -> ()")
_lib.define("prefill_bf16_nvfp4_lm(Tensor output_token, Tensor token_ids, Tensor embed_weight, Tensor layer_weights_packed, "
            "Tensor prefill_fused_weights_packed, Tensor final_norm_weight, Tensor lm_head_weight, "
            "Tensor lm_head_weight_packed, Tensor lm_head_scales, " + _PREFILL_BUFS +
            "Tensor proj_buf, Tensor proj_buf2, Tensor proj_buf_half, Tensor proj_act_packed, Tensor proj_act_scales, "
            "Tensor attn_buf, Tensor mlp_buf, Tensor dn_out_buf, Tensor beta_buf, Tensor alpha_buf, "
            "Tensor final_normed, Tensor hidden_bf16_out, Tensor lm_bmv, Tensor lm_bmi, "
            "Tensor lm_hidden_bf16, Tensor lm_hidden_packed, Tensor lm_hidden_scales, Tensor lm_logits_f16) -> ()")
_lib.define("prefill_megakernel_nvfp4(Tensor output_token, Tensor token_ids, " + _NVFP4_HEAD + _DECODE_TAIL +
            "int max_seq_len, int group_size) -> ()")
_lib.define("prefill_bf16_mega(Tensor output_token, Tensor token_ids, Tensor embed_weight, Tensor layer_weights_packed, "
            "Tensor final_norm_weight, Tensor lm_head_weight, " + _PREFILL_BUFS +
            "Tensor proj_buf, Tensor proj_buf2, Tensor attn_buf, Tensor mlp_buf, Tensor dn_out_buf, Tensor beta_buf, Tensor alpha_buf, "
            "Tensor final_normed, Tensor hidden_bf16_out, Tensor lm_bmv, Tensor lm_bmi) -> ()")
_lib.define("quantize_nvfp4_out(Tensor packed_out, Tensor scales_out, Tensor weight, int group_size) -> ()")
_lib.define("quantize_nvfp4_lm_out(Tensor packed_out, Tensor scales_out, Tensor weight) -> ()")


def _stream(t):
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _steps_args(embed, layers, final_norm, lm_head, k, v, dn, conv, hidden, out_token, position, max_seq_len, **kw):
    a = _capi.DecodeArgs()
    a.embed_weight = embed.data_ptr(); a.layer_weights = layers.data_ptr(); a.final_norm_weight = final_norm.data_ptr()
    a.lm_head_weight = lm_head.data_ptr(); a.fa_k_cache = k.data_ptr(); a.fa_v_cache = v.data_ptr()
    a.dn_states = dn.data_ptr(); a.conv_bufs = conv.data_ptr(); a.hidden_out = hidden.data_ptr()
    a.out_token = out_token.data_ptr(); a.position = position; a.max_seq_len = max_seq_len
    for key, val in kw.items():
        setattr(a, key, val)
    return a


def _decode(output_token, input_token_id, embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight,
            fa_k_cache, fa_v_cache, dn_states, conv_bufs, hidden_buffer, activations, residual, qkv_scratch, kv_scratch,
            attn_out, mlp_inter, z_scratch, beta_scratch, alpha_scratch, normalized, barrier_counter, barrier_generation,
            block_max_vals, block_max_idxs, lm_sync_counter, position, max_seq_len):
    with torch.cuda.device(output_token.device):
        _capi.check(_capi.lib().launch_decode(
            int(input_token_id), output_token.data_ptr(), embed_weight.data_ptr(), layer_weights_packed.data_ptr(),
            final_norm_weight.data_ptr(), lm_head_weight.data_ptr(), fa_k_cache.data_ptr(), fa_v_cache.data_ptr(),
            dn_states.data_ptr(), conv_bufs.data_ptr(), hidden_buffer.data_ptr(), *([None] * 15),
            int(position), int(max_seq_len), _stream(output_token)), "decode")


def _decode_nvfp4(output_token, input_token_id, embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight_packed,
                  lm_head_scales, lm_hidden_bf16, lm_hidden_packed, lm_hidden_scales, lm_logits_f16, fa_k_cache, fa_v_cache,
                  dn_states, conv_bufs, hidden_buffer, activations, residual, qkv_scratch, kv_scratch, attn_out, mlp_inter,
                  z_scratch, beta_scratch, alpha_scratch, normalized, barrier_counter, barrier_generation, block_max_vals,
                  block_max_idxs, lm_sync_counter, position, max_seq_len, group_size):
    if group_size != 32:
        raise RuntimeError("NVFP4 decode supports group_size 32")
    a = _steps_args(embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight_packed, fa_k_cache, fa_v_cache,
                    dn_states, conv_bufs, hidden_buffer, output_token, int(position), int(max_seq_len),
                    token_imm=int(input_token_id), n_steps=1)
    with torch.cuda.device(output_token.device):
        _capi.check(_capi.lib().qwen35_b200_decode_steps_nvfp4(C.byref(a), lm_head_scales.data_ptr(), _stream(output_token)), "decode_nvfp4")


def _decode_many_nvfp4(output_tokens, token_buffer, input_token_id, embed_weight, layer_weights_packed, final_norm_weight,
                       lm_head_weight_packed, lm_head_scales, lm_hidden_bf16, lm_hidden_packed, lm_hidden_scales, lm_logits_f16,
                       fa_k_cache, fa_v_cache, dn_states, conv_bufs, hidden_buffer, activations, residual, qkv_scratch,
                       kv_scratch, attn_out, mlp_inter, z_scratch, beta_scratch, alpha_scratch, normalized, barrier_counter,
                       barrier_generation, block_max_vals, block_max_idxs, lm_sync_counter, position, max_seq_len, group_size):
    if group_size != 32:
        raise RuntimeError("NVFP4 decode supports group_size 32")
    n = int(output_tokens.numel())
    a = _steps_args(embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight_packed, fa_k_cache, fa_v_cache,
                    dn_states, conv_bufs, hidden_buffer, token_buffer, int(position), int(max_seq_len),
                    token_imm=int(input_token_id), n_steps=n, out_tokens=output_tokens.data_ptr())
    with torch.cuda.device(output_tokens.device):
        _capi.check(_capi.lib().qwen35_b200_decode_steps_nvfp4(C.byref(a), lm_head_scales.data_ptr(), _stream(output_tokens)), "decode_many_nvfp4")


# The library keeps host copies of the device pointer tables, keyed by their addresses.  The reference's model.py packs
# its tables through torch's caching allocator, which readily hands the address of a freed table to the next one, so the
# address alone does not identify a table.  Every table TENSOR seen here is remembered by id with a weak reference; a
# tensor that was not seen before (a re-packed table, a rebuilt Decoder) makes the library drop its copies first.
_seen_tables = {}


def _note_table(t):
    if t is None:
        return
    key = id(t)
    ref = _seen_tables.get(key)
    if ref is not None and ref() is t:
        return
    for k in [k for k, r in _seen_tables.items() if r() is None]:
        del _seen_tables[k]
    import weakref
    _seen_tables[key] = weakref.ref(t)
    _capi.lib().qwen35_b200_forget_tables()


def _prefill_args(output_token, token_ids, embed_weight, layer_weights_packed, fused, final_norm_weight, lm_head_weight,
                  fa_k_cache, fa_v_cache, dn_states, conv_bufs, hidden, residual, normalized, proj_buf, proj_buf2, attn_buf,
                  mlp_buf, dn_out_buf, beta_buf, alpha_buf, final_normed, hidden_bf16_out, lm_bmv, lm_bmi):
    _note_table(layer_weights_packed)
    _note_table(fused)
    a = _capi.PrefillArgs()
    a.token_ids = token_ids.data_ptr(); a.seq_len = int(token_ids.size(0)); a.out_token = output_token.data_ptr()
    a.embed_weight = embed_weight.data_ptr(); a.layer_weights = layer_weights_packed.data_ptr()
    a.fused_layer_weights = None if fused is None else fused.data_ptr()
    a.final_norm_weight = final_norm_weight.data_ptr(); a.lm_head_weight = lm_head_weight.data_ptr()
    a.fa_k_cache = fa_k_cache.data_ptr(); a.fa_v_cache = fa_v_cache.data_ptr(); a.dn_states = dn_states.data_ptr(); a.conv_bufs = conv_bufs.data_ptr()
    a.hidden = hidden.data_ptr(); a.residual = residual.data_ptr(); a.normalized = normalized.data_ptr()
    a.proj_buf = proj_buf.data_ptr(); a.proj_buf2 = proj_buf2.data_ptr(); a.attn_buf = attn_buf.data_ptr(); a.mlp_buf = mlp_buf.data_ptr()
    a.dn_out_buf = dn_out_buf.data_ptr(); a.beta_buf = beta_buf.data_ptr(); a.alpha_buf = alpha_buf.data_ptr()
    a.final_normed = final_normed.data_ptr(); a.hidden_bf16_out = hidden_bf16_out.data_ptr(); a.lm_bmv = lm_bmv.data_ptr(); a.lm_bmi = lm_bmi.data_ptr()
    a.max_seq_len = int(fa_k_cache.size(2))
    return a


def _prefill_bf16(output_token, token_ids, embed_weight, layer_weights_packed, prefill_fused_weights_packed, final_norm_weight,
                  lm_head_weight, fa_k_cache, fa_v_cache, dn_states, conv_bufs, hidden, residual, normalized, proj_buf, proj_buf2,
                  proj_buf_half, proj_act_packed, proj_act_scales, attn_buf, mlp_buf, dn_out_buf, beta_buf, alpha_buf,
                  final_normed, hidden_bf16_out, lm_bmv, lm_bmi):
    a = _prefill_args(output_token, token_ids, embed_weight, layer_weights_packed, prefill_fused_weights_packed, final_norm_weight,
                      lm_head_weight, fa_k_cache, fa_v_cache, dn_states, conv_bufs, hidden, residual, normalized, proj_buf, proj_buf2,
                      attn_buf, mlp_buf, dn_out_buf, beta_buf, alpha_buf, final_normed, hidden_bf16_out, lm_bmv, lm_bmi)
    with torch.cuda.device(output_token.device):
        _capi.check(_capi.lib().qwen35_b200_prefill_bf16(C.byref(a), _stream(output_token)), "prefill_bf16")


def _prefill_bf16_nvfp4_lm(output_token, token_ids, embed_weight, layer_weights_packed, prefill_fused_weights_packed,
                           final_norm_weight, lm_head_weight, lm_head_weight_packed, lm_head_scales, fa_k_cache, fa_v_cache,
                           dn_states, conv_bufs, hidden, residual, normalized, proj_buf, proj_buf2, proj_buf_half, proj_act_packed,
                           proj_act_scales, attn_buf, mlp_buf, dn_out_buf, beta_buf, alpha_buf, final_normed, hidden_bf16_out,
                           lm_bmv, lm_bmi, lm_hidden_bf16, lm_hidden_packed, lm_hidden_scales, lm_logits_f16):
    a = _prefill_args(output_token, token_ids, embed_weight, layer_weights_packed, prefill_fused_weights_packed, final_norm_weight,
                      lm_head_weight, fa_k_cache, fa_v_cache, dn_states, conv_bufs, hidden, residual, normalized, proj_buf, proj_buf2,
                      attn_buf, mlp_buf, dn_out_buf, beta_buf, alpha_buf, final_normed, hidden_bf16_out, lm_bmv, lm_bmi)
    a.lm_head_weight_packed = lm_head_weight_packed.data_ptr(); a.lm_head_scales = lm_head_scales.data_ptr()
    with torch.cuda.device(output_token.device):
        _capi.check(_capi.lib().qwen35_b200_prefill_bf16(C.byref(a), _stream(output_token)), "prefill_bf16_nvfp4_lm")


def _prefill_megakernel_nvfp4(output_token, token_ids, embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight_packed,
                              lm_head_scales, lm_hidden_bf16, lm_hidden_packed, lm_hidden_scales, lm_logits_f16, fa_k_cache,
                              fa_v_cache, dn_states, conv_bufs, hidden_buffer, activations, residual, qkv_scratch, kv_scratch,
                              attn_out, mlp_inter, z_scratch, beta_scratch, alpha_scratch, normalized, barrier_counter,
                              barrier_generation, block_max_vals, block_max_idxs, lm_sync_counter, max_seq_len, group_size):
    """Token-serial prompt pass in one dispatch (reference: prefill_kernel_nvfp4, kernel_gb10_nvfp4.cu:1659-1755)."""
    if group_size != 32:
        raise RuntimeError("NVFP4 decode supports group_size 32")
    a = _steps_args(embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight_packed, fa_k_cache, fa_v_cache,
                    dn_states, conv_bufs, hidden_buffer, output_token, 0, int(max_seq_len),
                    forced_ids=token_ids.data_ptr(), n_steps=int(token_ids.size(0)), lm_last_only=1)
    with torch.cuda.device(output_token.device):
        _capi.check(_capi.lib().qwen35_b200_decode_steps_nvfp4(C.byref(a), lm_head_scales.data_ptr(), _stream(output_token)), "prefill_megakernel_nvfp4")


def _prefill_bf16_mega(output_token, token_ids, embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight, fa_k_cache,
                       fa_v_cache, dn_states, conv_bufs, hidden, residual, normalized, proj_buf, proj_buf2, attn_buf, mlp_buf,
                       dn_out_buf, beta_buf, alpha_buf, final_normed, hidden_bf16_out, lm_bmv, lm_bmi):
    """The reference's single-dispatch bf16 prompt pass (prefill_megakernel, prefill_megakernel.cu:840-1078).  It takes no
    fused-weight table, so the batched prefill runs with one tensor-core GEMM per matrix of the layer records."""
    a = _prefill_args(output_token, token_ids, embed_weight, layer_weights_packed, None, final_norm_weight,
                      lm_head_weight, fa_k_cache, fa_v_cache, dn_states, conv_bufs, hidden, residual, normalized, proj_buf, proj_buf2,
                      attn_buf, mlp_buf, dn_out_buf, beta_buf, alpha_buf, final_normed, hidden_bf16_out, lm_bmv, lm_bmi)
    with torch.cuda.device(output_token.device):
        _capi.check(_capi.lib().qwen35_b200_prefill_bf16(C.byref(a), _stream(output_token)), "prefill_bf16_mega")


def _quantize_nvfp4_out(packed_out, scales_out, weight, group_size):
    if weight.dtype != torch.bfloat16 or weight.dim() != 2 or not weight.is_contiguous():
        raise RuntimeError("weight must be a contiguous 2-D bfloat16 tensor")
    with torch.cuda.device(weight.device):
        _capi.check(_capi.lib().launch_quantize_nvfp4_out(weight.data_ptr(), int(weight.size(0)), int(weight.size(1)), int(group_size),
                                                          packed_out.data_ptr(), scales_out.data_ptr(), _stream(weight)), "quantize_nvfp4_out")


def _quantize_nvfp4_lm_out(packed_out, scales_out, weight):
    if weight.dtype != torch.bfloat16 or weight.dim() != 2 or not weight.is_contiguous():
        raise RuntimeError("weight must be a contiguous 2-D bfloat16 tensor")
    with torch.cuda.device(weight.device):
        _capi.check(_capi.lib().launch_quantize_nvfp4_lm_out(weight.data_ptr(), int(weight.size(0)), int(weight.size(1)),
                                                             packed_out.data_ptr(), scales_out.data_ptr(), _stream(weight)), "quantize_nvfp4_lm_out")


for _name, _fn in (("decode", _decode), ("decode_nvfp4", _decode_nvfp4), ("decode_many_nvfp4", _decode_many_nvfp4),
                   ("prefill_bf16", _prefill_bf16), ("prefill_bf16_nvfp4_lm", _prefill_bf16_nvfp4_lm),
                   ("prefill_megakernel_nvfp4", _prefill_megakernel_nvfp4), ("prefill_bf16_mega", _prefill_bf16_mega),
                   ("quantize_nvfp4_out", _quantize_nvfp4_out), ("quantize_nvfp4_lm_out", _quantize_nvfp4_lm_out)):
    _lib.impl(_name, _fn, "CUDA")
