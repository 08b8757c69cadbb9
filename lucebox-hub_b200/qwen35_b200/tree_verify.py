"""Host side of the tree-verify pass for the 27B-class hybrid target (the role of the reference's
models/qwen35_27b/src/qwen35_target_graph.cpp `TargetCache` + `build_qwen35_graph` and of the verify / accept / commit
loop of models/qwen35_27b/test/test_dflash.cpp).  PyTorch carries the device memory; all compute is in the C-ABI
library (qwen35_b200_tree_verify / _accept / _commit), which must be present: there is no fallback."""
import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _capi


@dataclass(frozen=True)
class TreeDims:
    n_layers: int
    hidden: int
    ffn: int
    vocab: int
    q_heads: int
    kv_heads: int
    dn_k_heads: int
    dn_v_heads: int
    head_dim: int = 256
    dn_dim: int = 128
    rot_dim: int = 64
    fa_period: int = 4
    rope_theta: float = 1.0e7
    rms_eps: float = 1.0e-6

    @property
    def conv_ch(self):
        return (2 * self.dn_k_heads + self.dn_v_heads) * self.dn_dim

    @property
    def fa_in(self):
        return (2 * self.q_heads + 2 * self.kv_heads) * self.head_dim

    @property
    def dn_in(self):
        return self.conv_ch + self.dn_v_heads * self.dn_dim

    def is_fa(self, il):
        return il % self.fa_period == self.fa_period - 1

    @property
    def n_fa(self):
        return sum(self.is_fa(i) for i in range(self.n_layers))

    @property
    def n_dn(self):
        return self.n_layers - self.n_fa


# dimensions of the reference's target (qwen35_target_graph.cpp:46-67, src/internal.h:116-130)
QWEN35_27B = TreeDims(n_layers=64, hidden=5120, ffn=17408, vocab=248320, q_heads=24, kv_heads=4, dn_k_heads=16, dn_v_heads=48)

MAX_NODES = 40
Q4K_BLOCK_BYTES = 144


def random_q4k(rows, cols, seed, device="cpu", sigma=0.02):
    """Random Q4_K super-blocks [rows, cols/256, 144] uint8 whose dequantised values have std ~ sigma and zero mean:
    uniform nibbles and 6-bit scales / mins, dmin = 7.5 * d (the mean nibble), d varied per block by +-25 %."""
    assert cols % 256 == 0
    nb = rows * (cols // 256)
    g = torch.Generator(device=device).manual_seed(seed)
    blocks = torch.randint(0, 256, (nb, Q4K_BLOCK_BYTES), dtype=torch.uint8, device=device, generator=g)
    # std of (sc*q - 7.5*m) for uniform sc, m in 0..63 and q in 0..15 is ~ 248.6
    d = (sigma / 248.6) * (0.75 + 0.5 * torch.rand(nb, device=device, generator=g))
    dh = d.to(torch.float16)
    dm = (7.5 * d).to(torch.float16)
    blocks[:, 0:2] = dh.view(torch.uint8).view(nb, 2)
    blocks[:, 2:4] = dm.view(torch.uint8).view(nb, 2)
    return blocks.view(rows, cols // 256, Q4K_BLOCK_BYTES)


def make_random_tree_weights(dims: TreeDims, seed: int, device="cpu"):
    """Seeded random weights in the layouts of Qwen35TreeLayer."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    D = dims

    def vec(n, mean, std):
        return (mean + std * torch.randn(n, generator=g)).float().to(device)

    layers = []
    for il in range(D.n_layers):
        s = seed * 1000 + il * 16
        L = {"attn_norm": vec(D.hidden, 1.0, 0.02), "post_norm": vec(D.hidden, 1.0, 0.02),
             "w_gate_up": random_q4k(2 * D.ffn, D.hidden, s + 1, device), "w_down": random_q4k(D.hidden, D.ffn, s + 2, device)}
        if D.is_fa(il):
            L["w_in"] = random_q4k(D.fa_in, D.hidden, s + 3, device)
            L["w_out"] = random_q4k(D.hidden, D.q_heads * D.head_dim, s + 4, device)
            L["q_norm"] = vec(D.head_dim, 1.0, 0.02)
            L["k_norm"] = vec(D.head_dim, 1.0, 0.02)
        else:
            L["w_in"] = random_q4k(D.dn_in, D.hidden, s + 3, device)
            L["w_out"] = random_q4k(D.hidden, D.dn_v_heads * D.dn_dim, s + 4, device)
            L["w_ba"] = (0.02 * torch.randn(2 * D.dn_v_heads, D.hidden, generator=g)).bfloat16().to(device)
            L["conv_w"] = (0.2 * torch.randn(D.conv_ch, 4, generator=g)).float().to(device)
            L["ssm_a"] = (-torch.exp(torch.log(0.5 + 15.5 * torch.rand(D.dn_v_heads, generator=g)))).float().to(device)
            L["dt_bias"] = vec(D.dn_v_heads, 1.0, 0.02)
            L["ssm_norm"] = vec(D.dn_dim, 1.0, 0.02)
        layers.append(L)
    return {"layers": layers, "token_embd": random_q4k(D.vocab, D.hidden, seed * 1000 + 999, device),
            "output_norm": vec(D.hidden, 1.0, 0.02), "output_w": random_q4k(D.vocab, D.hidden, seed * 1000 + 998, device)}


def random_tree(n_nodes, max_depth, seed):
    """Seeded random parent array in DFS (pre-order) numbering: parents[t] < t, children contiguous in pre-order."""
    rng = np.random.default_rng(seed)
    parents, depth, stack = [-1], [0], [0]           # stack = current root-to-node path
    while len(parents) < n_nodes:
        # attach the next node to a random node of the current path (keeps pre-order numbering), respecting max depth
        cand = [i for i, nd in enumerate(stack) if depth[nd] < max_depth]
        if not cand:
            stack = stack[:1]
            continue
        k = cand[-1] if rng.random() < 0.6 else int(rng.choice(cand))      # mostly extend the chain, sometimes branch
        stack = stack[:k + 1]
        parents.append(stack[-1]); depth.append(depth[stack[-1]] + 1)
        stack.append(len(parents) - 1)
    return parents


KV_TYPES = {"bf16": 0, "q8_0": 1, "q4_0": 2, "f16": 3}       # the library's kv_type codes
KV_BLOCK_BYTES = {"q8_0": 34, "q4_0": 18}                    # bytes per 32-element block of the quantised types


class TreeTarget:
    """Caches, weights table and scratch of one target model instance on one GPU."""

    def __init__(self, dims: TreeDims, weights, max_ctx: int, device="cuda", max_nodes: int = MAX_NODES, capture_layers=(), feat_cap: int = 0,
                 kv_type: str = "bf16"):
        """kv_type: "bf16", or one of the reference's K / V cache types (qwen35_target_graph.cpp:110-122): "q8_0" (its
        default; uint8 [n_fa, kv_heads, max_ctx, 272]), "q4_0" (uint8 [..., 144]) or "f16"; rows are converted in the
        kernel when a node is written and read back as bf16 operands.
        capture_layers / feat_cap: keep the outputs of those layers in a ring of feat_cap positions for the draft
        (`target_feat`, bf16 [feat_cap, len(capture_layers) * hidden]; the reference's target captures layers 1, 16, 31, 46, 61)."""
        self.dims, self.max_ctx, self.max_nodes = dims, int(max_ctx), int(max_nodes)
        self.device = torch.device(device)
        self._lib = _capi.lib()
        self._w = weights
        D = dims
        self._dims_c = _capi.TreeDimsC(D.n_layers, D.hidden, D.ffn, D.vocab, D.q_heads, D.kv_heads, D.head_dim, D.dn_k_heads, D.dn_v_heads, D.dn_dim,
                                       D.rot_dim, D.fa_period, D.rope_theta, D.rms_eps)
        self._layers_c = (_capi.TreeLayerC * D.n_layers)()
        # a matrix given as bf16 [rows, cols] instead of Q4_K super-blocks (uint8 [rows, cols/256, 144]) is flagged dense
        mat_bit = {"w_in": 1, "w_out": 2, "w_gate_up": 4, "w_down": 8}
        for il, L in enumerate(weights["layers"]):
            mask = 0
            for k, v in L.items():
                assert v.is_cuda and v.is_contiguous(), k
                setattr(self._layers_c[il], k, v.data_ptr())
                if k in mat_bit:
                    assert v.dtype in (torch.uint8, torch.bfloat16), k
                    mask |= mat_bit[k] if v.dtype == torch.bfloat16 else 0
            self._layers_c[il].dense_mask = mask
        self._dense_mask = (1 if weights["token_embd"].dtype == torch.bfloat16 else 0) | (2 if weights["output_w"].dtype == torch.bfloat16 else 0)
        dev = self.device
        if kv_type not in KV_TYPES:
            raise ValueError("kv_type must be one of %s" % (sorted(KV_TYPES),))
        self.kv_type = kv_type
        if kv_type in KV_BLOCK_BYTES:
            self.k_cache = torch.zeros(max(D.n_fa, 1), D.kv_heads, self.max_ctx, D.head_dim // 32 * KV_BLOCK_BYTES[kv_type], dtype=torch.uint8, device=dev)
        else:
            self.k_cache = torch.zeros(max(D.n_fa, 1), D.kv_heads, self.max_ctx, D.head_dim,
                                       dtype=torch.float16 if kv_type == "f16" else torch.bfloat16, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.ssm_state = torch.zeros(max(D.n_dn, 1), D.dn_v_heads, D.dn_dim, D.dn_dim, dtype=torch.float32, device=dev)
        self.conv_state = torch.zeros(max(D.n_dn, 1), 3, D.conv_ch, dtype=torch.float32, device=dev)
        self.node_states = torch.zeros(max(D.n_dn, 1), self.max_nodes, D.dn_v_heads, D.dn_dim, D.dn_dim, dtype=torch.float16, device=dev)
        self.node_conv = torch.zeros(max(D.n_dn, 1), self.max_nodes, D.conv_ch, dtype=torch.float32, device=dev)
        self.node_argmax = torch.zeros(64, dtype=torch.int32, device=dev)
        self.path = torch.zeros(64, dtype=torch.int32, device=dev)
        self.result = torch.zeros(2, dtype=torch.int32, device=dev)
        nbytes = self._lib.qwen35_b200_tree_scratch_bytes(C.byref(self._dims_c), self.max_nodes, self.max_ctx)
        self._scratch = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self.past = 0
        self._tokens = self._parents = None
        self._n = 0
        self.capture_layers = tuple(int(x) for x in capture_layers)
        if len(self.capture_layers) > 8:
            raise ValueError("at most 8 capture layers")
        self.feat_cap = int(feat_cap) if self.capture_layers else 0
        self.target_feat = (torch.zeros(self.feat_cap, len(self.capture_layers) * D.hidden, dtype=torch.bfloat16, device=dev)
                            if self.feat_cap > 0 else None)

    def _args(self, n, **kw):
        a = _capi.TreeVerifyArgs()
        a.dims = self._dims_c
        a.layers = C.cast(self._layers_c, C.POINTER(_capi.TreeLayerC))
        a.token_embd = self._w["token_embd"].data_ptr(); a.output_norm = self._w["output_norm"].data_ptr(); a.output_w = self._w["output_w"].data_ptr()
        a.n_nodes = n; a.max_nodes = self.max_nodes
        a.node_tokens = self._tokens.data_ptr() if self._tokens is not None else None
        a.parents = self._parents.data_ptr() if self._parents is not None else None
        a.past = self.past; a.max_ctx = self.max_ctx
        a.k_cache = self.k_cache.data_ptr(); a.v_cache = self.v_cache.data_ptr()
        a.ssm_state = self.ssm_state.data_ptr(); a.conv_state = self.conv_state.data_ptr()
        a.node_states = self.node_states.data_ptr(); a.node_conv = self.node_conv.data_ptr()
        a.node_argmax = self.node_argmax.data_ptr()
        a.scratch = self._scratch.data_ptr(); a.scratch_bytes = self._scratch.numel()
        a.dense_mask = self._dense_mask
        a.kv_type = KV_TYPES[self.kv_type]
        if self.target_feat is not None:
            a.target_feat = self.target_feat.data_ptr(); a.feat_cap = self.feat_cap; a.n_capture = len(self.capture_layers)
            for i, il in enumerate(self.capture_layers):
                a.capture_layers[i] = il
        for k, v in kw.items():
            setattr(a, k, _capi.ptr(v) if torch.is_tensor(v) else v)
        return a

    def _stream(self):
        return C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def verify(self, tokens, parents, **kw):
        """Evaluate the tree (int32 tensors on the device, DFS order).  Returns the per-node arg-max tokens (GPU)."""
        self._tokens = tokens.to(self.device, torch.int32).contiguous()
        self._parents = parents.to(self.device, torch.int32).contiguous()
        self._n = int(self._tokens.numel())
        with torch.cuda.device(self.device):
            _capi.check(self._lib.qwen35_b200_tree_verify(C.byref(self._args(self._n, **kw)), self._stream()), "tree_verify")
        return self.node_argmax[:self._n]

    def accept(self):
        """Walk the verified tree on the device.  Returns (path tensor, result tensor [length, next token]) on the GPU."""
        with torch.cuda.device(self.device):
            _capi.check(self._lib.qwen35_b200_tree_accept(self._tokens.data_ptr(), self._parents.data_ptr(), self.node_argmax.data_ptr(), self._n,
                                                          self.path.data_ptr(), self.result.data_ptr(), self._stream()), "tree_accept")
        return self.path, self.result

    def commit(self, path=None, result=None):
        """Commit the accepted path (default: the one accept() found).  One device->host read of the accepted length
        keeps the host's `past` in step."""
        path = self.path if path is None else path
        result = self.result if result is None else result
        with torch.cuda.device(self.device):
            _capi.check(self._lib.qwen35_b200_tree_commit(C.byref(self._args(self._n)), path.data_ptr(), result.data_ptr(), self._stream()), "tree_commit")
        n_acc = int(result[0].item())
        self.past += n_acc
        return n_acc

    def feature_window(self, n_last: int):
        """The last `n_last` committed positions of the feature ring in position order, bf16 [n, n_capture * hidden]:
        what the draft takes as target_hidden_cat (test_dflash.cpp:1097-1120 copies the same window out of the ring)."""
        if self.target_feat is None:
            raise ValueError("no feature ring: construct with capture_layers and feat_cap")
        n = min(int(n_last), self.past, self.feat_cap)
        idx = (torch.arange(self.past - n, self.past, device=self.device) % self.feat_cap)
        return self.target_feat.index_select(0, idx)

    def check_status(self):
        _capi.check(self._lib.qwen35_b200_status(None), "status")


def dequant_q4k(blocks: torch.Tensor, want="f32"):
    """GPU dequantisation of Q4_K super-blocks [..., 144] uint8 -> [..., 256] f32 or bf16."""
    lib = _capi.lib()
    b = blocks.contiguous().view(-1, Q4K_BLOCK_BYTES)
    out = torch.empty(b.shape[0], 256, dtype=torch.float32 if want == "f32" else torch.bfloat16, device=b.device)
    with torch.cuda.device(b.device):
        _capi.check(lib.qwen35_b200_dequant_q4k(b.data_ptr(), b.shape[0], out.data_ptr() if want == "f32" else None,
                                                out.data_ptr() if want != "f32" else None,
                                                C.c_void_p(torch.cuda.current_stream(b.device).cuda_stream)), "dequant_q4k")
    return out.view(*blocks.shape[:-1], 256)
