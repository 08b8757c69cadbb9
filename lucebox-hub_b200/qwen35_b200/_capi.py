"""ctypes view of libqwen35_b200.so (declarations: include/qwen35_b200.h).

There is no fallback: if the library is missing or a call fails, an exception is raised.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# QWEN35_B200_LIB selects another build of the same library (kernel experiments); the default is the in-tree build
LIB_PATH = os.environ.get("QWEN35_B200_LIB") or os.path.join(_HERE, "libqwen35_b200.so")

OK = 0
STATUS_NAMES = {0: "ok", 1: "device wait timed out", 2: "bad argument", 3: "CUDA error", 4: "unsupported"}


class Qwen35Error(RuntimeError):
    pass


class DecodeArgs(C.Structure):
    _fields_ = [
        ("embed_weight", C.c_void_p), ("layer_weights", C.c_void_p),
        ("final_norm_weight", C.c_void_p), ("lm_head_weight", C.c_void_p),
        ("fa_k_cache", C.c_void_p), ("fa_v_cache", C.c_void_p),
        ("dn_states", C.c_void_p), ("conv_bufs", C.c_void_p),
        ("token_in", C.c_void_p), ("token_imm", C.c_int),
        ("forced_ids", C.c_void_p), ("out_token", C.c_void_p), ("out_tokens", C.c_void_p),
        ("logits_out", C.c_void_p), ("hidden_out", C.c_void_p), ("dbg_hidden", C.c_void_p), ("dbg_teacher", C.c_void_p),
        ("position", C.c_int), ("max_seq_len", C.c_int), ("n_steps", C.c_int), ("lm_last_only", C.c_int), ("dbg_num_layers", C.c_int), ("dbg_time", C.c_void_p), ("dbg_time_cta", C.c_int),
    ]


class PrefillArgs(C.Structure):
    _fields_ = [
        ("token_ids", C.c_void_p), ("seq_len", C.c_int), ("out_token", C.c_void_p),
        ("embed_weight", C.c_void_p), ("layer_weights", C.c_void_p), ("fused_layer_weights", C.c_void_p),
        ("final_norm_weight", C.c_void_p), ("lm_head_weight", C.c_void_p),
        ("fa_k_cache", C.c_void_p), ("fa_v_cache", C.c_void_p), ("dn_states", C.c_void_p), ("conv_bufs", C.c_void_p),
        ("hidden", C.c_void_p), ("residual", C.c_void_p), ("normalized", C.c_void_p),
        ("proj_buf", C.c_void_p), ("proj_buf2", C.c_void_p), ("attn_buf", C.c_void_p), ("mlp_buf", C.c_void_p),
        ("dn_out_buf", C.c_void_p), ("beta_buf", C.c_void_p), ("alpha_buf", C.c_void_p),
        ("final_normed", C.c_void_p), ("hidden_bf16_out", C.c_void_p), ("lm_bmv", C.c_void_p), ("lm_bmi", C.c_void_p),
        ("logits_out", C.c_void_p), ("max_seq_len", C.c_int), ("dbg_num_layers", C.c_int),
        ("lm_head_weight_packed", C.c_void_p), ("lm_head_scales", C.c_void_p),
        ("dbg_teacher", C.c_void_p), ("dbg_hidden", C.c_void_p),
    ]


class BatchedArgs(C.Structure):
    _fields_ = [
        ("batch", C.c_int), ("max_ctx", C.c_int), ("num_pages", C.c_int), ("max_pages", C.c_int),
        ("tokens_in", C.c_void_p), ("tokens_out", C.c_void_p), ("positions", C.c_void_p), ("block_table", C.c_void_p),
        ("embed_weight", C.c_void_p), ("layer_weights", C.c_void_p), ("fused_layer_weights", C.c_void_p),
        ("final_norm_weight", C.c_void_p), ("lm_head_weight", C.c_void_p),
        ("k_pages", C.c_void_p), ("v_pages", C.c_void_p), ("dn_states", C.c_void_p), ("conv_bufs", C.c_void_p),
        ("logits_out", C.c_void_p), ("dbg_hidden", C.c_void_p), ("dbg_teacher", C.c_void_p),
        ("advance_positions", C.c_int), ("dbg_num_layers", C.c_int),
        ("layer_weights_host", C.c_void_p), ("fused_layer_weights_host", C.c_void_p),
        ("scratch", C.c_void_p), ("scratch_bytes", C.c_size_t),
    ]


class TreeDimsC(C.Structure):
    _fields_ = [(k, C.c_int) for k in ("n_layers", "hidden", "ffn", "vocab", "q_heads", "kv_heads", "head_dim", "dn_k_heads", "dn_v_heads",
                                        "dn_dim", "rot_dim", "fa_period")] + [("rope_theta", C.c_float), ("rms_eps", C.c_float)]


class TreeLayerC(C.Structure):
    _fields_ = [(k, C.c_void_p) for k in ("attn_norm", "post_norm", "w_in", "w_ba", "w_out", "w_gate_up", "w_down", "q_norm", "k_norm", "conv_w",
                                           "ssm_a", "dt_bias", "ssm_norm")] + [("dense_mask", C.c_ulonglong), ("r1", C.c_void_p), ("r2", C.c_void_p)]


class TreeVerifyArgs(C.Structure):
    _fields_ = [
        ("dims", TreeDimsC), ("layers", C.POINTER(TreeLayerC)), ("token_embd", C.c_void_p), ("output_norm", C.c_void_p), ("output_w", C.c_void_p),
        ("n_nodes", C.c_int), ("max_nodes", C.c_int), ("node_tokens", C.c_void_p), ("parents", C.c_void_p), ("past", C.c_int), ("max_ctx", C.c_int),
        ("k_cache", C.c_void_p), ("v_cache", C.c_void_p), ("ssm_state", C.c_void_p), ("conv_state", C.c_void_p), ("node_states", C.c_void_p),
        ("node_conv", C.c_void_p), ("node_argmax", C.c_void_p), ("logits_out", C.c_void_p), ("dbg_hidden", C.c_void_p), ("dbg_num_layers", C.c_int),
        ("scratch", C.c_void_p), ("scratch_bytes", C.c_size_t), ("dbg_teacher", C.c_void_p), ("dense_mask", C.c_uint),
        ("target_feat", C.c_void_p), ("feat_cap", C.c_int), ("n_capture", C.c_int), ("capture_layers", C.c_int * 8), ("kv_type", C.c_int),
    ]


class DraftDimsC(C.Structure):
    _fields_ = [(k, C.c_int) for k in ("hidden", "n_layers", "n_heads", "n_kv_heads", "head_dim", "inter", "n_target_layers", "q_len")] + \
               [("eps", C.c_float), ("rope_theta", C.c_float)]


class DraftLayerC(C.Structure):
    _fields_ = [(k, C.c_void_p) for k in ("attn_norm", "wq", "wkv", "q_norm", "k_norm", "wo", "ffn_norm", "w_gate_up", "w_down")]


class DraftArgs(C.Structure):
    _fields_ = [
        ("dims", DraftDimsC), ("layers", C.POINTER(DraftLayerC)), ("fc", C.c_void_p), ("hidden_norm", C.c_void_p), ("out_norm", C.c_void_p),
        ("noise_embed", C.c_void_p), ("target_hidden_cat", C.c_void_p), ("ctx_len", C.c_int), ("hidden_out", C.c_void_p), ("lm_head", C.c_void_p),
        ("lm_head_q4k", C.c_int), ("vocab", C.c_int), ("logits_out", C.c_void_p), ("scratch", C.c_void_p), ("scratch_bytes", C.c_size_t),
        ("stream", C.c_void_p),
    ]


_lib = None

# name -> (restype, argtypes); every symbol include/qwen35_b200.h declares
_vp, _i = C.c_void_p, C.c_int
SIGNATURES = {
    "launch_decode": (_i, [_i, _vp] + [_vp] * 8 + [_vp] * 11 + [_vp] * 5 + [_i, _i, _vp]),
    "qwen35_b200_decode_steps": (_i, [C.POINTER(DecodeArgs), _vp]),
    "qwen35_b200_decode_steps_nvfp4": (_i, [C.POINTER(DecodeArgs), _vp, _vp]),
    "launch_decode_nvfp4": (_i, [_vp, _vp] + [_vp] * 5 + [_vp] * 4 + [_vp] * 5 + [_vp] * 10 + [_vp] * 5 + [_i, _i, _i, _vp]),
    "launch_decode_many_nvfp4": (_i, [_vp, _vp, _i] + [_vp] * 5 + [_vp] * 4 + [_vp] * 5 + [_vp] * 10 + [_vp] * 5 + [_i, _i, _i, _vp]),
    "qwen35_b200_decode_steps_static": (_i, [C.POINTER(DecodeArgs), _vp]),
    "qwen35_b200_prefill_bf16": (_i, [C.POINTER(PrefillArgs), _vp]),
    "launch_prefill_bf16_nvfp4_lm": (_i, [_vp, _i, _vp] + [_vp] * 7 + [_vp] * 4 + [_vp] * 3 + [_vp] * 5 + [_vp] * 5 + [_vp] * 4 + [_vp] * 4 + [_vp]),
    "launch_prefill_bf16": (_i, [_vp, _i, _vp] + [_vp] * 5 + [_vp] * 4 + [_vp] * 3 + [_vp] * 5 + [_vp] * 5 + [_vp] * 4 + [_vp]),
    "launch_prefill_bf16_mega": (_i, [_vp, _i, _vp] + [_vp] * 4 + [_vp] * 4 + [_vp] * 3 + [_vp] * 4 + [_vp] * 3 + [_vp] * 4 + [_vp]),
    "launch_prefill_megakernel_nvfp4": (_i, [_vp, _i, _vp] + [_vp] * 5 + [_vp] * 4 + [_vp] * 5 + [_vp] * 10 + [_vp] * 5 + [_i, _i, _vp]),
    "launch_quantize_nvfp4_out": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp]),
    "launch_quantize_nvfp4_lm_out": (_i, [_vp, _i, _i, _vp, _vp, _vp]),
    "qwen35_b200_decode_batched": (_i, [C.POINTER(BatchedArgs), _vp]),
    "qwen35_b200_batched_scratch_bytes": (C.c_size_t, [_i, _i]),
    "qwen35_b200_forget_tables": (None, []),
    "qwen35_b200_draft_topk": (_i, [_vp, _i, _i, _i, C.c_float, _vp, _vp, _vp]),
    "qwen35_b200_build_ddtree": (_i, [_vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "qwen35_b200_draft_scratch_bytes": (C.c_size_t, [C.POINTER(DraftDimsC), _i]),
    "qwen35_b200_draft_forward": (_i, [C.POINTER(DraftArgs)]),
    "qwen35_b200_tree_scratch_bytes": (C.c_size_t, [C.POINTER(TreeDimsC), _i, _i]),
    "qwen35_b200_tree_verify": (_i, [C.POINTER(TreeVerifyArgs), _vp]),
    "qwen35_b200_tree_accept": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp]),
    "qwen35_b200_tree_commit": (_i, [C.POINTER(TreeVerifyArgs), _vp, _vp, _vp]),
    "qwen35_b200_dequant_q4k": (_i, [_vp, C.c_size_t, _vp, _vp, _vp]),
    "qwen35_b200_gemm_bf16": (_i, [_vp, _i, _vp, _i, _vp, _i, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "qwen35_b200_gemm_q4k": (_i, [_vp, _i, _vp, _i, _vp, _i, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "qwen35_b200_nvfp4_act_bytes": (C.c_size_t, [_i, _i, C.POINTER(C.c_size_t)]),
    "qwen35_b200_quantize_act_nvfp4": (_i, [_vp, _i, _i, _vp, _vp, _vp]),
    "qwen35_b200_gemm_nvfp4": (_i, [_vp, _vp, _i, _vp, _vp, _i, _i, C.c_float, _vp, _i, _i, _vp, _i, _vp]),
    "qwen35_b200_status": (_i, [_vp]),
    "qwen35_b200_clear_status": (_i, [_vp]),
    "qwen35_b200_workspace_if_any": (_vp, []),
    "qwen35_b200_debug_read": (_i, [_i, _vp]),
    "qwen35_b200_rope_inv_freq": (_i, [C.POINTER(C.c_float)]),
    "qwen35_b200_launch_count": (C.c_longlong, []),
    "qwen35_b200_last_error": (C.c_char_p, []),
}


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise Qwen35Error(
                f"{LIB_PATH} is missing: build it with `python lucebox-hub_b200/build.py` "
                "(there is no CPU or PyTorch fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int, what: str):
    if status != OK:
        msg = lib().qwen35_b200_last_error().decode()
        raise Qwen35Error(f"{what}: status {status} ({STATUS_NAMES.get(status, '?')}): {msg}")


def ptr(t):
    return None if t is None else t.data_ptr()
