"""Host side of the DFlash draft forward (the role of the reference's `DraftWeights` / `build_draft_graph`,
models/qwen35_27b/src/qwen3_dflash_graph.cpp:38-166 and src/internal.h): a 5-layer non-causal block-diffusion model that
proposes `q_len` tokens from the target's captured features.  PyTorch carries the device memory; all compute is in the
C-ABI library (qwen35_b200_draft_forward), which must be present: there is no fallback."""
import ctypes as C
from dataclasses import dataclass

import torch

from . import _capi


@dataclass(frozen=True)
class DraftDims:
    hidden: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    inter: int
    head_dim: int = 128
    n_target_layers: int = 5
    q_len: int = 16
    eps: float = 1.0e-6
    rope_theta: float = 1.0e7

    @property
    def q_dim(self):
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self):
        return self.n_kv_heads * self.head_dim


# dimensions of the reference's draft (include/dflash27b.h:26-39)
DFLASH_27B = DraftDims(hidden=5120, n_layers=5, n_heads=32, n_kv_heads=8, inter=17408)

LAYER_MATRICES = ("wq", "wkv", "wo", "w_gate_up", "w_down")
LAYER_VECTORS = ("attn_norm", "q_norm", "k_norm", "ffn_norm")


def make_random_draft_weights(dims: DraftDims, seed: int, device="cpu", sigma: float = 0.02):
    """Seeded random-init weights in the layout the library takes: bf16 [out][in] matrices (wkv = [wk ; wv],
    w_gate_up = [w_gate ; w_up]), f32 norm vectors around 1."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)       # drawn on `device` (a CPU draw of the full-size model takes minutes)
    H, D = dims.hidden, dims

    def mat(o, i):
        return (torch.randn(o, i, generator=g, device=dev) * sigma).bfloat16()

    def vec(n):
        return (1.0 + 0.1 * torch.randn(n, generator=g, device=dev)).float()

    w = {"fc": mat(H, D.n_target_layers * H), "hidden_norm": vec(H), "out_norm": vec(H), "layers": []}
    for _ in range(D.n_layers):
        w["layers"].append({
            "attn_norm": vec(H), "wq": mat(D.q_dim, H), "wkv": mat(2 * D.kv_dim, H), "q_norm": vec(D.head_dim), "k_norm": vec(D.head_dim),
            "wo": mat(H, D.q_dim), "ffn_norm": vec(H), "w_gate_up": mat(2 * D.inter, H), "w_down": mat(H, D.inter),
        })
    return w


def draft_weights_to(w, device):
    out = {k: (v.to(device) if torch.is_tensor(v) else v) for k, v in w.items() if k != "layers"}
    out["layers"] = [{k: v.to(device) for k, v in L.items()} for L in w["layers"]]
    return out


class DraftModel:
    """forward(noise_embed [q_len, hidden] bf16, target_hidden_cat [ctx_len, 5*hidden] bf16) -> hidden_out [q_len, hidden] bf16,
    and logits [q_len, vocab] bf16 when an LM head (the target's: bf16 matrix or Q4_K blocks) is attached."""

    def __init__(self, dims: DraftDims, weights, max_ctx: int, device="cuda", lm_head=None, lm_head_q4k=False, vocab=0):
        self.dims, self.w, self.max_ctx, self.device = dims, weights, max_ctx, torch.device(device)
        self._lib = _capi.lib()
        self._dims_c = _capi.DraftDimsC(dims.hidden, dims.n_layers, dims.n_heads, dims.n_kv_heads, dims.head_dim, dims.inter, dims.n_target_layers,
                                        dims.q_len, dims.eps, dims.rope_theta)
        self._layers_c = (_capi.DraftLayerC * dims.n_layers)()
        for i, L in enumerate(weights["layers"]):
            for k in ("attn_norm", "wq", "wkv", "q_norm", "k_norm", "wo", "ffn_norm", "w_gate_up", "w_down"):
                t = L[k]
                assert t.is_cuda and t.is_contiguous(), k
                setattr(self._layers_c[i], k, t.data_ptr())
        nbytes = int(self._lib.qwen35_b200_draft_scratch_bytes(C.byref(self._dims_c), max_ctx))
        if nbytes == 0:
            raise ValueError("draft dims not supported by the library")
        self._scratch = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        self.lm_head, self.lm_head_q4k, self.vocab = lm_head, bool(lm_head_q4k), int(vocab)

    def forward(self, noise_embed: torch.Tensor, target_hidden_cat: torch.Tensor):
        D = self.dims
        ctx = 0 if target_hidden_cat is None else int(target_hidden_cat.shape[0])
        if ctx > self.max_ctx:
            raise ValueError(f"ctx_len {ctx} > max_ctx {self.max_ctx}")
        assert noise_embed.shape == (D.q_len, D.hidden) and noise_embed.dtype == torch.bfloat16 and noise_embed.is_contiguous()
        if ctx:
            assert target_hidden_cat.shape[1] == D.n_target_layers * D.hidden and target_hidden_cat.dtype == torch.bfloat16
            assert target_hidden_cat.is_contiguous()
        out = torch.empty(D.q_len, D.hidden, dtype=torch.bfloat16, device=self.device)
        logits = torch.empty(D.q_len, self.vocab, dtype=torch.bfloat16, device=self.device) if self.lm_head is not None else None
        a = _capi.DraftArgs()
        a.dims, a.layers = self._dims_c, self._layers_c
        a.fc, a.hidden_norm, a.out_norm = self.w["fc"].data_ptr(), self.w["hidden_norm"].data_ptr(), self.w["out_norm"].data_ptr()
        a.noise_embed = noise_embed.data_ptr()
        a.target_hidden_cat = target_hidden_cat.data_ptr() if ctx else None
        a.ctx_len = ctx
        a.hidden_out = out.data_ptr()
        if self.lm_head is not None:
            a.lm_head, a.lm_head_q4k, a.vocab, a.logits_out = self.lm_head.data_ptr(), int(self.lm_head_q4k), self.vocab, logits.data_ptr()
        a.scratch, a.scratch_bytes = self._scratch.data_ptr(), self._scratch.numel()
        with torch.cuda.device(self.device):
            a.stream = torch.cuda.current_stream().cuda_stream
            _capi.check(self._lib.qwen35_b200_draft_forward(C.byref(a)), "draft_forward")
        return (out, logits) if logits is not None else out

    def check_status(self):
        with torch.cuda.device(self.device):
            _capi.check(self._lib.qwen35_b200_status(C.c_void_p(torch.cuda.current_stream().cuda_stream)), "device status")
