"""Decode API for the B200 Qwen3.5-0.8B kernels -- a drop-in for the reference's
`models/qwen35_0p8b/model.py`.

Same names and meaning as the reference: the dimension constants (model.py:7-42), the
`weights` dict (`embed_weight`, `final_norm_weight`, `lm_head_weight`, `layer_data`,
model.py:386-391), `_pack_layer_weights` (128-byte layer records, model.py:410-427) and
`class Decoder` with `step`, `step_many`, `prefill_tokens`, `reset`, `generate`
(model.py:473-817).  State tensors have the reference's shapes and layouts so callers that
reach into `_fa_k_cache`, `_dn_states`, `_conv_bufs`, `_hidden` keep working.

Differences: `max_seq_len` is a constructor argument (the reference fixes 2048); `step_many`
and `prefill_tokens` also work for the BF16 backend; with no checkpoint available weights
come from `qwen35_b200.weights.make_random_weights`.  There is no CPU fallback: every call
goes to libqwen35_b200.so and raises if it is missing or reports an error.
"""
from __future__ import annotations

import ctypes as C
import struct

import torch

from . import _capi
from .config import MAX_SEQ_LEN, QWEN35_0P8B

_D = QWEN35_0P8B
NUM_LAYERS = _D.num_layers
HIDDEN_SIZE = _D.hidden
INTERMEDIATE_SIZE = _D.intermediate
VOCAB_SIZE = _D.vocab
FA_NUM_Q_HEADS = _D.fa_q_heads
FA_NUM_KV_HEADS = _D.fa_kv_heads
FA_HEAD_DIM = _D.fa_head_dim
FA_Q_SIZE = _D.fa_q_size
FA_QPROJ_SIZE = _D.fa_qproj_size
FA_KV_SIZE = _D.fa_kv_size
DN_NUM_HEADS = _D.dn_heads
DN_KEY_DIM = _D.dn_key_dim
DN_VALUE_DIM = _D.dn_value_dim
DN_QK_SIZE = _D.dn_qk_size
DN_V_SIZE = _D.dn_v_size
DN_CONV_CHANNELS = _D.dn_conv_channels
DN_CONV_KERNEL = _D.dn_conv_kernel
LAYER_TYPE = _D.layer_types


def load_weights(model_name="random:1234", verbose=True, backend="bf16", device="cuda"):
    """Reference signature (model.py:314-319).  `random:<seed>` gives the seeded random-init weights; a path to a
    HuggingFace checkpoint directory or `.safetensors` file is read directly (no network, no tokenizer: the second
    return value is None).  A hub id cannot be resolved where this runs."""
    import os

    from .weights import load_safetensors_weights, make_random_weights, weights_to
    name = str(model_name)
    if name.startswith("random:"):
        return weights_to(make_random_weights(int(name.split(":", 1)[1]), _D), device), None
    if os.path.exists(name):
        return load_safetensors_weights(name, _D, device), None
    raise FileNotFoundError(f"{name}: not 'random:<seed>' and not a local checkpoint path (no hub download is possible here)")


NVFP4_GROUP_SIZE = 32
NVFP4_LM_GROUP_SIZE = 16
NVFP4_TC_ROWS_PER_TILE = 128
NVFP4_TC_K_PER_TILE = 64


def _check_bf16_matrix(weight):
    if weight.dtype != torch.bfloat16:
        raise TypeError(f"expected bfloat16 weight, got {weight.dtype}")
    if weight.dim() != 2:
        raise ValueError(f"expected 2D weight, got shape {tuple(weight.shape)}")


def _quantize_matrix_nvfp4(weight, group_size=NVFP4_GROUP_SIZE):
    """Decode-body NVFP4 layout (reference model.py:100-114): {"packed": u8 [rows, cols/2], "scales": f16 [rows, cols/group]}."""
    _check_bf16_matrix(weight)
    rows, cols = weight.shape
    if cols % 2 != 0 or cols % group_size != 0:
        raise ValueError(f"in_dim {cols} must be divisible by 2 and group_size {group_size}")
    w = weight.contiguous()
    packed = torch.empty((rows, cols // 2), dtype=torch.uint8, device=w.device)
    scales = torch.empty((rows, cols // group_size), dtype=torch.float16, device=w.device)
    with torch.cuda.device(w.device):
        _capi.check(_capi.lib().launch_quantize_nvfp4_out(w.data_ptr(), rows, cols, group_size, packed.data_ptr(), scales.data_ptr(),
                                                          C.c_void_p(torch.cuda.current_stream(w.device).cuda_stream)), "quantize_nvfp4_out")
    return {"packed": packed, "scales": scales}


def _quantize_matrix_nvfp4_lm(weight):
    """Tensor-core NVFP4 layout (reference model.py:117-134): 16-element blocks, swizzled E4M3 scales."""
    _check_bf16_matrix(weight)
    rows, cols = weight.shape
    if rows % 128 != 0:
        raise ValueError(f"lm_head out_dim {rows} must be divisible by 128")
    if cols % 64 != 0:
        raise ValueError(f"lm_head in_dim {cols} must be divisible by 64")
    w = weight.contiguous()
    packed = torch.empty((rows, cols // 2), dtype=torch.uint8, device=w.device)
    scales = torch.zeros((rows // 128) * (cols // 64) * 512, dtype=torch.uint8, device=w.device)
    with torch.cuda.device(w.device):
        _capi.check(_capi.lib().launch_quantize_nvfp4_lm_out(w.data_ptr(), rows, cols, packed.data_ptr(), scales.data_ptr(),
                                                             C.c_void_p(torch.cuda.current_stream(w.device).cuda_stream)), "quantize_nvfp4_lm_out")
    return {"packed": packed, "scales": scales}


def _quantize_matrix_nvfp4_tc(weight, padded_rows=None):
    """The same layout for a matrix whose row count is padded with zero rows to a multiple of 128
    (reference model.py:137-168)."""
    _check_bf16_matrix(weight)
    rows, cols = weight.shape
    if cols % NVFP4_TC_K_PER_TILE != 0:
        raise ValueError(f"in_dim {cols} must be divisible by {NVFP4_TC_K_PER_TILE}")
    if padded_rows is None:
        padded_rows = ((rows + NVFP4_TC_ROWS_PER_TILE - 1) // NVFP4_TC_ROWS_PER_TILE) * NVFP4_TC_ROWS_PER_TILE
    if padded_rows < rows or padded_rows % NVFP4_TC_ROWS_PER_TILE != 0:
        raise ValueError(f"padded_rows {padded_rows} must be a multiple of 128 and >= rows {rows}")
    src = weight
    if padded_rows != rows:
        src = torch.zeros((padded_rows, cols), dtype=weight.dtype, device=weight.device)
        src[:rows].copy_(weight)
    out = _quantize_matrix_nvfp4_lm(src)
    out.update(rows=rows, padded_rows=padded_rows)
    return out


def _attach_nvfp4_weights(weights, group_size=NVFP4_GROUP_SIZE, verbose=False):
    """Quantise the decode-hot matrices (reference model.py:206-311): per layer qkv/z/out/gate/up/down (DeltaNet) or
    q/k/v/o/gate/up/down (attention) in the decode-body layout, the LM head in the tensor-core layout."""
    if "nvfp4" in weights and weights["nvfp4"]["group_size"] == group_size:
        return weights
    layers = []
    for ld in weights["layer_data"]:
        p = ld["ptrs"]
        q = lambda t: _quantize_matrix_nvfp4(t, group_size)   # noqa: E731
        if ld["type"] == 1:
            qs = [q(p[1]), q(p[2]), q(p[3]), q(p[6]), q(p[8]), q(p[9]), q(p[10])]
            ptrs = [p[0], qs[0]["packed"], qs[0]["scales"], qs[1]["packed"], qs[1]["scales"], qs[2]["packed"], qs[2]["scales"],
                    p[4], p[5], qs[3]["packed"], qs[3]["scales"], p[7],
                    qs[4]["packed"], qs[4]["scales"], qs[5]["packed"], qs[5]["scales"], qs[6]["packed"], qs[6]["scales"]]
        else:
            qs = [q(p[1]), q(p[2]), q(p[9]), q(p[11]), q(p[12]), q(p[13])]
            ptrs = [p[0], qs[0]["packed"], qs[0]["scales"], qs[1]["packed"], qs[1]["scales"],
                    p[3], p[4], p[5], p[6], p[7], p[8], qs[2]["packed"], qs[2]["scales"], p[10],
                    qs[3]["packed"], qs[3]["scales"], qs[4]["packed"], qs[4]["scales"], qs[5]["packed"], qs[5]["scales"]]
        layers.append({"type": ld["type"], "ptrs": ptrs, "quantized": qs})
    lm = _quantize_matrix_nvfp4_lm(weights["lm_head_weight"])
    weights["nvfp4"] = {"group_size": group_size, "lm_group_size": NVFP4_LM_GROUP_SIZE, "layer_data": layers,
                        "lm_head_weight_packed": lm["packed"], "lm_head_scales": lm["scales"]}
    return weights


def _pack_layer_weights_nvfp4(layer_data, group_size, device="cuda"):
    """Device blob of records {int type; int group_size; int pad[2]; void* ptrs[24]} (reference model.py:430-447)."""
    rec = 16 + 24 * 8
    buf = bytearray(len(layer_data) * rec)
    for i, ld in enumerate(layer_data):
        struct.pack_into("iiii", buf, i * rec, ld["type"], group_size, 0, 0)
        for j, t in enumerate(ld["ptrs"]):
            struct.pack_into("Q", buf, i * rec + 16 + j * 8, t.data_ptr())
    return torch.frombuffer(buf, dtype=torch.uint8).to(device)


DN_PROJ_FUSED_SIZE = DN_CONV_CHANNELS + DN_V_SIZE + 2 * DN_NUM_HEADS
DN_PROJ_FUSED_PADDED_SIZE = ((DN_PROJ_FUSED_SIZE + 127) // 128) * 128
PREFILL_PROJ_FUSED_SIZE = max(DN_PROJ_FUSED_PADDED_SIZE, FA_QPROJ_SIZE + 2 * FA_KV_SIZE, INTERMEDIATE_SIZE * 2)
PREFILL_PROJ_SCRATCH_SIZE = max(DN_CONV_CHANNELS, FA_QPROJ_SIZE, INTERMEDIATE_SIZE)


def _attach_prefill_fused_weights(weights):
    """Concatenated projection and gate/up matrices per layer (reference model.py:171-189)."""
    if "prefill_fused_layer_data" in weights:
        return
    fused = []
    for ld in weights["layer_data"]:
        p = ld["ptrs"]
        if ld["type"] == 1:
            proj = torch.cat([p[1], p[2], p[3]], dim=0).contiguous()
            gate_up = torch.cat([p[8], p[9]], dim=0).contiguous()
        else:
            proj = torch.cat([p[1], p[2], p[3], p[4]], dim=0).contiguous()
            gate_up = torch.cat([p[11], p[12]], dim=0).contiguous()
        fused.append({"proj_weight": proj, "gate_up_weight": gate_up})
    weights["prefill_fused_layer_data"] = fused


def _attach_prefill_nvfp4_weights(weights, verbose=False):
    """NVFP4 (tensor-core layout) copies of the two fused prompt matrices of every layer (reference model.py:190-215): the
    DeltaNet projection padded to 8320 rows, gate/up as it is.  With them in the fused table the prompt pass runs those two
    GEMMs block-scaled on FP4 operands."""
    _attach_prefill_fused_weights(weights)
    fused = weights["prefill_fused_layer_data"]
    if fused and "proj_weight_packed" in fused[0]:
        return weights
    for ld, f in zip(weights["layer_data"], fused):
        rows = DN_PROJ_FUSED_PADDED_SIZE if ld["type"] == 0 else f["proj_weight"].shape[0]
        pq = _quantize_matrix_nvfp4_tc(f["proj_weight"], padded_rows=rows)
        gq = _quantize_matrix_nvfp4_tc(f["gate_up_weight"])
        f["proj_weight_packed"], f["proj_weight_scales"] = pq["packed"], pq["scales"]
        f["gate_up_weight_packed"], f["gate_up_weight_scales"] = gq["packed"], gq["scales"]
    return weights


def _pack_prefill_fused_layer_weights(fused_layer_data, device="cuda", with_nvfp4=True):
    """Device blob of 6-pointer records (reference model.py:450-470): bf16 projection and gate/up, then the packed / scales
    pairs of their NVFP4 copies (null when the weights carry none, or with_nvfp4=False)."""
    _capi.lib().qwen35_b200_forget_tables()       # a new table may reuse the address of a freed one
    buf = bytearray(len(fused_layer_data) * 48)
    for i, ld in enumerate(fused_layer_data):
        q = [ld[k].data_ptr() if (with_nvfp4 and k in ld) else 0
             for k in ("proj_weight_packed", "proj_weight_scales", "gate_up_weight_packed", "gate_up_weight_scales")]
        struct.pack_into("QQQQQQ", buf, i * 48, ld["proj_weight"].data_ptr(), ld["gate_up_weight"].data_ptr(), *q)
    return torch.frombuffer(buf, dtype=torch.uint8).to(device)


def _pack_layer_weights(layer_data, device="cuda"):
    """Device blob of 24 records {int type; int pad[3]; void* ptrs[14]} (model.py:410-427)."""
    if str(device) != "cpu":
        _capi.lib().qwen35_b200_forget_tables()   # a new table may reuse the address of a freed one
    ptr_size, max_ptrs, header = 8, 14, 16
    rec = header + max_ptrs * ptr_size
    buf = bytearray(len(layer_data) * rec)
    for i, ld in enumerate(layer_data):
        off = i * rec
        struct.pack_into("iiii", buf, off, ld["type"], 0, 0, 0)
        for j, t in enumerate(ld["ptrs"]):
            if t.dtype != torch.bfloat16 or not t.is_contiguous():
                raise TypeError("layer tensors must be contiguous bf16")
            struct.pack_into("Q", buf, off + header + j * ptr_size, t.data_ptr())
    return torch.frombuffer(buf, dtype=torch.uint8).to(device)


class Decoder:
    """Stateful greedy decoder, batch 1 (reference: model.py:473)."""

    def __init__(self, weights=None, tokenizer=None, model_name="random:1234", backend="bf16",
                 verbose=False, max_seq_len=MAX_SEQ_LEN, device="cuda", prefill_nvfp4=False):
        """prefill_nvfp4=True: the batched prompt pass runs its fused projection and gate/up GEMMs and the LM head block-scaled
        on NVFP4 operands (the reference's tensor-core prompt option, prefill.cu:1210-1262 + prefill_bf16_nvfp4_lm)."""
        if backend not in ("bf16", "nvfp4", "auto", None):
            raise ValueError(f"unsupported backend: {backend}")
        self.backend = "nvfp4" if backend == "nvfp4" else "bf16"
        self.backend_label = "NVFP4 decode" if self.backend == "nvfp4" else "BF16"
        self._nvfp4_group_size = NVFP4_GROUP_SIZE
        self._lib = _capi.lib()
        self.device = torch.device(device)
        if weights is None:
            weights, tokenizer = load_weights(model_name, verbose=verbose, device=device)
        self.tokenizer = tokenizer
        self.max_seq_len = int(max_seq_len)
        self._position = 0
        self._weights = weights
        self._embed_weight = weights["embed_weight"]
        self._final_norm_weight = weights["final_norm_weight"]
        self._lm_head_weight = weights["lm_head_weight"]
        self._layer_weights_packed = _pack_layer_weights(weights["layer_data"], device)
        self.prefill_nvfp4 = bool(prefill_nvfp4)
        if self.prefill_nvfp4:
            _attach_prefill_nvfp4_weights(weights)
            if "prefill_lm_nvfp4" not in weights:
                weights["prefill_lm_nvfp4"] = _quantize_matrix_nvfp4_lm(weights["lm_head_weight"])
            self._prefill_lm_packed, self._prefill_lm_scales = weights["prefill_lm_nvfp4"]["packed"], weights["prefill_lm_nvfp4"]["scales"]
        else:
            _attach_prefill_fused_weights(weights)
        self._prefill_fused_weights_packed = _pack_prefill_fused_layer_weights(weights["prefill_fused_layer_data"], device, with_nvfp4=self.prefill_nvfp4)
        self._prefill_buffers = None
        self._prefill_buffer_tokens = 0
        self._layer_weights_packed_nvfp4 = None
        if self.backend == "nvfp4":
            _attach_nvfp4_weights(weights, self._nvfp4_group_size)
            nv = weights["nvfp4"]
            self._layer_weights_packed_nvfp4 = _pack_layer_weights_nvfp4(nv["layer_data"], nv["group_size"], device)
            self._lm_head_weight_packed = nv["lm_head_weight_packed"]
            self._lm_head_scales = nv["lm_head_scales"]

        dev = self.device
        n_fa = sum(1 for t in LAYER_TYPE if t == 1)
        n_dn = NUM_LAYERS - n_fa
        self._fa_k_cache = torch.zeros(n_fa, FA_NUM_KV_HEADS, self.max_seq_len, FA_HEAD_DIM, dtype=torch.bfloat16, device=dev)
        self._fa_v_cache = torch.zeros_like(self._fa_k_cache)
        # [layer][head][v][k] f32 -- value-major like the reference kernels (kernel.cu:684)
        self._dn_states = torch.zeros(n_dn, DN_NUM_HEADS, DN_VALUE_DIM, DN_KEY_DIM, dtype=torch.float32, device=dev)
        self._conv_bufs = torch.zeros(n_dn, DN_CONV_CHANNELS, DN_CONV_KERNEL, dtype=torch.float32, device=dev)
        self._hidden = torch.empty(HIDDEN_SIZE, dtype=torch.bfloat16, device=dev)
        self._out_token = torch.zeros(1, dtype=torch.int32, device=dev)
        # step(): the kernel stores the token straight into pinned host memory (same address on the device under unified
        # addressing), so reading it back costs a stream synchronisation and no copy call; the argument tuple is built once
        self._out_token_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._out_token_view = self._out_token_host.numpy()
        self._step_args = None
        self._token_buf = torch.zeros(1, dtype=torch.int32, device=dev)

    # ---- helpers ---------------------------------------------------------------------------
    def _stream(self):
        return C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def _args(self, **kw):
        a = _capi.DecodeArgs()
        a.embed_weight = self._embed_weight.data_ptr()
        a.layer_weights = self._layer_weights_packed.data_ptr()
        a.final_norm_weight = self._final_norm_weight.data_ptr()
        a.lm_head_weight = self._lm_head_weight.data_ptr()
        a.fa_k_cache = self._fa_k_cache.data_ptr()
        a.fa_v_cache = self._fa_v_cache.data_ptr()
        a.dn_states = self._dn_states.data_ptr()
        a.conv_bufs = self._conv_bufs.data_ptr()
        a.hidden_out = self._hidden.data_ptr()
        a.out_token = self._out_token.data_ptr()
        a.position = self._position
        a.max_seq_len = self.max_seq_len
        for k, v in kw.items():
            setattr(a, k, v)
        return a

    def _run(self, a):
        with torch.cuda.device(self.device):
            if self.backend == "nvfp4":
                a.layer_weights = self._layer_weights_packed_nvfp4.data_ptr()
                a.lm_head_weight = self._lm_head_weight_packed.data_ptr()
                _capi.check(self._lib.qwen35_b200_decode_steps_nvfp4(C.byref(a), self._lm_head_scales.data_ptr(), self._stream()), "decode_nvfp4")
            else:
                _capi.check(self._lib.qwen35_b200_decode_steps(C.byref(a), self._stream()), "decode")

    def check_status(self):
        """Synchronise and raise if a kernel recorded an error (e.g. a bounded wait ran out)."""
        with torch.cuda.device(self.device):
            _capi.check(self._lib.qwen35_b200_status(self._stream()), "device status")

    # ---- reference API -----------------------------------------------------------------------
    def step(self, token_id: int) -> int:
        """Decode one token, return the next token id (model.py:678-714; one D2H sync)."""
        if self.backend == "nvfp4":
            self._run(self._args(token_imm=int(token_id), n_steps=1))
            self._position += 1
            return int(self._out_token.item())
        if self._step_args is None:
            none = None
            self._step_args = (self._out_token_host.data_ptr(),
                               self._embed_weight.data_ptr(), self._layer_weights_packed.data_ptr(),
                               self._final_norm_weight.data_ptr(), self._lm_head_weight.data_ptr(),
                               self._fa_k_cache.data_ptr(), self._fa_v_cache.data_ptr(),
                               self._dn_states.data_ptr(), self._conv_bufs.data_ptr(),
                               self._hidden.data_ptr(), *([none] * 10), *([none] * 5))
            self._step_dev = torch.device(self.device)
            self._step_dev_index = self._step_dev.index if self._step_dev.index is not None else torch.cuda.current_device()
        if torch.cuda.current_device() != self._step_dev_index:
            torch.cuda.set_device(self._step_dev_index)
        stream = torch.cuda.current_stream(self._step_dev)
        _capi.check(self._lib.launch_decode(int(token_id), *self._step_args, self._position, self.max_seq_len,
                                            C.c_void_p(stream.cuda_stream)), "launch_decode")
        self._position += 1
        stream.synchronize()
        return int(self._out_token_view[0])

    def step_many(self, token_id: int, num_steps: int, logits_out=None, dbg_time=None, dbg_time_cta=0) -> torch.Tensor:
        """`num_steps` greedy steps in one launch, tokens fed back on the device
        (model.py:716-743 offers this for NVFP4 only).  Returns int32 [num_steps] on the GPU."""
        if num_steps < 0:
            raise ValueError("num_steps must be non-negative")
        out = torch.empty(num_steps, dtype=torch.int32, device=self.device)
        if num_steps == 0:
            return out
        a = self._args(token_imm=int(token_id), n_steps=num_steps, out_tokens=out.data_ptr(),
                       logits_out=_capi.ptr(logits_out), dbg_time=_capi.ptr(dbg_time), dbg_time_cta=dbg_time_cta)
        self._run(a)
        self._position += num_steps
        return out

    def _ensure_prefill_buffers(self, max_tokens: int):
        """Scratch of the batched prefill, sizes of the reference (model.py:569-602)."""
        if self._prefill_buffers is not None and self._prefill_buffer_tokens >= max_tokens:
            return self._prefill_buffers
        bf16 = dict(dtype=torch.bfloat16, device=self.device)
        f32 = dict(dtype=torch.float32, device=self.device)
        self._prefill_buffers = dict(
            hidden=torch.empty(max_tokens * HIDDEN_SIZE, **bf16),
            residual=torch.empty(max_tokens * HIDDEN_SIZE, **bf16),
            normalized=torch.empty(max_tokens * HIDDEN_SIZE, **bf16),
            proj_buf=torch.empty(max_tokens * PREFILL_PROJ_FUSED_SIZE, **bf16),
            proj_buf2=torch.empty(max_tokens * PREFILL_PROJ_SCRATCH_SIZE, **bf16),
            attn_buf=torch.empty(max_tokens * max(FA_Q_SIZE, FA_KV_SIZE), **bf16),
            mlp_buf=torch.empty(max_tokens * INTERMEDIATE_SIZE, **bf16),
            dn_out_buf=torch.empty(max_tokens * DN_V_SIZE, **bf16),
            beta_buf=torch.empty(max_tokens * DN_NUM_HEADS, **f32),
            alpha_buf=torch.empty(max_tokens * DN_NUM_HEADS, **f32),
            final_normed=torch.empty(HIDDEN_SIZE, **bf16),
            hidden_bf16_out=torch.empty(HIDDEN_SIZE, **bf16),
            lm_bmv=torch.empty(1024, **f32),
            lm_bmi=torch.empty(1024, dtype=torch.int32, device=self.device),
        )
        self._prefill_buffer_tokens = max_tokens
        return self._prefill_buffers

    def prefill_tokens(self, token_ids: torch.Tensor, logits_out=None, mode="batched", dbg_num_layers=0,
                       dbg_teacher=None, dbg_hidden=None) -> int:
        """Reset, run the prompt, return the first generated token (reference model.py:745-799).
        mode="batched": tensor-core GEMMs + chunk-64 gated delta rule + causal attention (the
        reference's prefill_bf16 op).  mode="serial": the decode megakernel token by token (the
        reference's token-serial `prefill_megakernel`, kernel_gb10_nvfp4.cu:1659-1755).  mode="mega": the
        batched pass without the fused-weight table, one GEMM per matrix (the reference's prefill_bf16_mega op)."""
        if token_ids.device.type != "cuda" or token_ids.dtype != torch.int32 or token_ids.dim() != 1:
            raise TypeError("token_ids must be a 1D CUDA int32 tensor")
        self.reset()
        n = int(token_ids.numel())
        if n == 0:
            raise ValueError("empty prompt")
        if mode == "serial":
            a = self._args(forced_ids=token_ids.data_ptr(), n_steps=n, lm_last_only=1, logits_out=_capi.ptr(logits_out))
            self._run(a)
        else:
            b = self._ensure_prefill_buffers(n)
            a = _capi.PrefillArgs()
            a.token_ids = token_ids.data_ptr(); a.seq_len = n; a.out_token = self._out_token.data_ptr()
            a.embed_weight = self._embed_weight.data_ptr(); a.layer_weights = self._layer_weights_packed.data_ptr()
            a.fused_layer_weights = None if mode == "mega" else self._prefill_fused_weights_packed.data_ptr()
            a.final_norm_weight = self._final_norm_weight.data_ptr(); a.lm_head_weight = self._lm_head_weight.data_ptr()
            a.fa_k_cache = self._fa_k_cache.data_ptr(); a.fa_v_cache = self._fa_v_cache.data_ptr()
            a.dn_states = self._dn_states.data_ptr(); a.conv_bufs = self._conv_bufs.data_ptr()
            for k in ("hidden", "residual", "normalized", "proj_buf", "proj_buf2", "attn_buf", "mlp_buf", "dn_out_buf",
                      "beta_buf", "alpha_buf", "final_normed", "hidden_bf16_out", "lm_bmv", "lm_bmi"):
                setattr(a, k, b[k].data_ptr())
            a.logits_out = _capi.ptr(logits_out); a.max_seq_len = self.max_seq_len; a.dbg_num_layers = dbg_num_layers
            a.dbg_teacher = _capi.ptr(dbg_teacher); a.dbg_hidden = _capi.ptr(dbg_hidden)
            if self.prefill_nvfp4 and mode != "mega":
                a.lm_head_weight_packed = self._prefill_lm_packed.data_ptr(); a.lm_head_scales = self._prefill_lm_scales.data_ptr()
            with torch.cuda.device(self.device):
                _capi.check(self._lib.qwen35_b200_prefill_bf16(C.byref(a), self._stream()), "prefill_bf16")
            self._hidden.copy_(b["hidden_bf16_out"])
        self._position = n
        return int(self._out_token.item())

    def forced_steps(self, token_ids: torch.Tensor, logits_out=None, dbg_hidden=None, dbg_teacher=None,
                     dbg_num_layers=0) -> torch.Tensor:
        """Teacher-forced decode: feed `token_ids` one per step, return the arg-max of every step."""
        n = int(token_ids.numel())
        out = torch.empty(n, dtype=torch.int32, device=self.device)
        a = self._args(forced_ids=token_ids.data_ptr(), n_steps=n, out_tokens=out.data_ptr(),
                       logits_out=_capi.ptr(logits_out), dbg_hidden=_capi.ptr(dbg_hidden),
                       dbg_teacher=_capi.ptr(dbg_teacher), dbg_num_layers=dbg_num_layers)
        self._run(a)
        self._position += n
        return out

    def debug_read(self, which: str) -> torch.Tensor:
        """Inter-stage vector of the library workspace (bf16, CPU): 'xa', 'o', 'h1', 'm', 'h2'."""
        idx, n = {"xa": (0, 8224), "o": (1, 2048), "h1": (2, 1024), "m": (3, 3584), "h2": (4, 1024)}[which]
        out = torch.empty(n, dtype=torch.bfloat16)
        with torch.cuda.device(self.device):
            _capi.check(self._lib.qwen35_b200_debug_read(idx, out.data_ptr()), "debug_read")
        return out

    def reset(self):
        self._position = 0
        self._fa_k_cache.zero_()
        self._fa_v_cache.zero_()
        self._dn_states.zero_()
        self._conv_bufs.zero_()

    def generate(self, prompt, max_tokens: int = 100):
        """Greedy generation.  `prompt` is a string when a tokenizer is attached (reference
        behaviour, model.py:804-817) or a sequence of token ids; returns text or ids."""
        if isinstance(prompt, str):
            if self.tokenizer is None:
                raise RuntimeError("no tokenizer attached; pass token ids")
            ids = self.tokenizer.encode(prompt, add_special_tokens=True)
        else:
            ids = [int(t) for t in prompt]
        first = self.prefill_tokens(torch.tensor(ids, dtype=torch.int32, device=self.device))
        out = [first]
        if max_tokens > 1:
            out += self.step_many(first, max_tokens - 1).tolist()
        if isinstance(prompt, str):
            eos = self.tokenizer.eos_token_id
            if eos in out:
                out = out[:out.index(eos)]
            return self.tokenizer.decode(out, skip_special_tokens=True)
        return out


KV_PAGE = 64


class BatchedDecoder:
    """`batch` independent sequences decoded together on one GPU (the benchmark configuration "64 sequences per GPU").
    Each sequence owns its DeltaNet state, conv window and KV pages; weights are shared.  Prefill a sequence with
    `prefill(seq, ids)` (runs the bs=1 batched-prefill kernels into that sequence's slots), then `step()` advances
    every sequence by one greedy token."""

    def __init__(self, weights, batch, max_ctx=2304, device="cuda", groups=1):
        """groups > 1: a graph step runs the batch as that many equal sub-batches on concurrent streams, each call with its own
        scratch.  Results are identical to one batch; measured on B200 at 64 sequences x 2048 tokens it is slower (2.26 ms
        per step as one batch, 2.49 ms as two sub-batches, 3.19 ms as four: the kernels already fill the SMs and the
        weights are read once per sub-batch), so the default is one batch."""
        self._lib = _capi.lib()
        self.device = torch.device(device)
        self.batch = int(batch)
        self.groups = int(groups) if int(batch) % max(int(groups), 1) == 0 else 1
        self.max_ctx = int(max_ctx)
        self.max_pages = (self.max_ctx + KV_PAGE - 1) // KV_PAGE
        self.num_pages = self.batch * self.max_pages
        self._weights = weights
        _attach_prefill_fused_weights(weights)
        self._layer_weights_packed = _pack_layer_weights(weights["layer_data"], device)
        self._prefill_fused_weights_packed = _pack_prefill_fused_layer_weights(weights["prefill_fused_layer_data"], device, with_nvfp4=False)
        # host copies of the two tables: with them a step never synchronises
        self._graph = None; self._warm = False
        self._layer_weights_host = self._layer_weights_packed.cpu()
        self._fused_weights_host = self._prefill_fused_weights_packed.cpu()
        dev = self.device
        self.k_pages = torch.zeros(6, self.num_pages, FA_NUM_KV_HEADS, KV_PAGE, FA_HEAD_DIM, dtype=torch.bfloat16, device=dev)
        self.v_pages = torch.zeros_like(self.k_pages)
        self.dn_states = torch.zeros(self.batch, 18, DN_NUM_HEADS, DN_VALUE_DIM, DN_KEY_DIM, dtype=torch.float32, device=dev)
        self.conv_bufs = torch.zeros(self.batch, 18, DN_CONV_CHANNELS, DN_CONV_KERNEL, dtype=torch.float32, device=dev)
        # sequence b owns pages [b*max_pages, (b+1)*max_pages): the identity table of an unfragmented pool
        self.block_table = torch.arange(self.num_pages, dtype=torch.int32, device=dev).view(self.batch, self.max_pages).contiguous()
        self.positions = torch.zeros(self.batch, dtype=torch.int32, device=dev)
        self.tokens = torch.zeros(self.batch, dtype=torch.int32, device=dev)
        self._out = torch.zeros(self.batch, dtype=torch.int32, device=dev)
        self._one = None
        # Positions advance on the device; the host keeps an upper bound on the largest one (every step adds one) so that a
        # step or a graph replay that would write past max_ctx is refused here.  A caller that writes `positions` directly
        # is still covered by the kernels' own check, which skips the sequence and sets the status word.
        self._max_position = 0
        self._streams, self._group_scratch = [], []
        if self.groups > 1:
            nb = self._lib.qwen35_b200_batched_scratch_bytes(self.batch // self.groups, self.max_ctx)
            for _ in range(self.groups):
                self._streams.append(torch.cuda.Stream(device=dev))
                self._group_scratch.append(torch.empty(nb, dtype=torch.uint8, device=dev))

    def load_sequence(self, seq, k_cache, v_cache, dn_states, conv_bufs, position, next_token):
        """Install a prefilled bs=1 state ([6,2,L,256] caches, [18,16,128,128] state, [18,6144,4] conv) as sequence `seq`."""
        L = int(position)
        kp = self.k_pages[:, seq * self.max_pages:(seq + 1) * self.max_pages]        # [6, pages, 2, 64, 256]
        vp = self.v_pages[:, seq * self.max_pages:(seq + 1) * self.max_pages]
        pad = self.max_pages * KV_PAGE
        kk = torch.zeros(6, FA_NUM_KV_HEADS, pad, FA_HEAD_DIM, dtype=torch.bfloat16, device=self.device)
        vv = torch.zeros_like(kk)
        kk[:, :, :L] = k_cache[:, :, :L]
        vv[:, :, :L] = v_cache[:, :, :L]
        kp.copy_(kk.view(6, FA_NUM_KV_HEADS, self.max_pages, KV_PAGE, FA_HEAD_DIM).permute(0, 2, 1, 3, 4))
        vp.copy_(vv.view(6, FA_NUM_KV_HEADS, self.max_pages, KV_PAGE, FA_HEAD_DIM).permute(0, 2, 1, 3, 4))
        self.dn_states[seq].copy_(dn_states)
        self.conv_bufs[seq].copy_(conv_bufs)
        self.positions[seq] = L
        self.tokens[seq] = int(next_token)
        self._max_position = max(self._max_position, L)

    def prefill(self, seq, token_ids):
        """Prefill one sequence with the bs=1 prefill path and install it."""
        if self._one is None:
            self._one = Decoder(weights=self._weights, max_seq_len=self.max_pages * KV_PAGE, device=self.device)
        first = self._one.prefill_tokens(token_ids)
        self.load_sequence(seq, self._one._fa_k_cache, self._one._fa_v_cache, self._one._dn_states, self._one._conv_bufs,
                           int(token_ids.numel()), first)
        return first

    def _args(self, **kw):
        a = _capi.BatchedArgs()
        a.batch = self.batch; a.max_ctx = self.max_ctx; a.num_pages = self.num_pages; a.max_pages = self.max_pages
        a.tokens_in = self.tokens.data_ptr(); a.tokens_out = self._out.data_ptr(); a.positions = self.positions.data_ptr()
        a.block_table = self.block_table.data_ptr()
        a.embed_weight = self._weights["embed_weight"].data_ptr(); a.layer_weights = self._layer_weights_packed.data_ptr()
        a.fused_layer_weights = self._prefill_fused_weights_packed.data_ptr()
        a.layer_weights_host = self._layer_weights_host.data_ptr(); a.fused_layer_weights_host = self._fused_weights_host.data_ptr()
        a.final_norm_weight = self._weights["final_norm_weight"].data_ptr(); a.lm_head_weight = self._weights["lm_head_weight"].data_ptr()
        a.k_pages = self.k_pages.data_ptr(); a.v_pages = self.v_pages.data_ptr()
        a.dn_states = self.dn_states.data_ptr(); a.conv_bufs = self.conv_bufs.data_ptr()
        a.advance_positions = 1
        for k, v in kw.items():
            setattr(a, k, v)
        return a

    def _launch(self, a):
        with torch.cuda.device(self.device):
            _capi.check(self._lib.qwen35_b200_decode_batched(C.byref(a), C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)),
                        "decode_batched")
            self.tokens.copy_(self._out)

    def _group_args(self, g):
        """Arguments of sub-batch g: the same pools, this group's rows of every per-sequence array, its own scratch."""
        a = self._args()
        n = self.batch // self.groups
        first = g * n
        a.batch = n
        a.tokens_in = self.tokens[first:].data_ptr(); a.tokens_out = self._out[first:].data_ptr()
        a.positions = self.positions[first:].data_ptr(); a.block_table = self.block_table[first:].data_ptr()
        a.dn_states = self.dn_states[first:].data_ptr(); a.conv_bufs = self.conv_bufs[first:].data_ptr()
        a.scratch = self._group_scratch[g].data_ptr(); a.scratch_bytes = self._group_scratch[g].numel()
        return a

    def _launch_groups(self):
        """Fork the current stream into one stream per sub-batch, join, then hand the new tokens over (capturable)."""
        with torch.cuda.device(self.device):
            cur = torch.cuda.current_stream(self.device)
            for g, st in enumerate(self._streams):
                st.wait_stream(cur)
                with torch.cuda.stream(st):
                    _capi.check(self._lib.qwen35_b200_decode_batched(C.byref(self._group_args(g)), C.c_void_p(st.cuda_stream)), "decode_batched")
            for st in self._streams:
                cur.wait_stream(st)
            self.tokens.copy_(self._out)

    def step(self, graph=False, **kw):
        """One greedy token for every sequence; the new tokens become the next step's inputs.  Returns int32 [batch]
        (GPU; the same buffer every step: clone it to keep a value).  graph=True replays a CUDA graph of the step's
        launches (recorded on the second such call: the first runs eagerly so the library's scratch exists)."""
        if self._max_position + 1 > self.max_ctx:
            raise ValueError(f"batched decode: a sequence is at position {self._max_position}, the cache holds max_ctx = {self.max_ctx} tokens")
        if kw.get("advance_positions", 1):
            self._max_position += 1
        if graph and not kw:
            if self._graph is None and self._warm:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.device(self.device), torch.cuda.graph(g):
                    if self.groups > 1:
                        self._launch_groups()
                    else:
                        self._launch(self._args())
                self._graph = g
            if self._graph is not None:
                self._graph.replay()
                return self.tokens
        self._launch(self._args(**{k: (_capi.ptr(v) if torch.is_tensor(v) else v) for k, v in kw.items()}))
        self._warm = True
        return self.tokens

    def check_status(self):
        with torch.cuda.device(self.device):
            _capi.check(self._lib.qwen35_b200_status(C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)), "device status")
