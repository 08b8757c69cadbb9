"""Python face of the draft-tree entry points (qwen35_b200_draft_topk, qwen35_b200_build_ddtree): the tree that
qwen35_b200.tree_verify.TreeTarget.verify takes, built as the reference's driver builds it
(models/qwen35_27b/test/test_dflash.cpp:143-390)."""
import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _capi


def draft_topk(logits: torch.Tensor, k: int, temperature: float = 1.0):
    """logits f32 [n_positions, vocab] on the GPU -> (log_probs f32 [n, k], token ids int32 [n, k]) on the GPU."""
    assert logits.is_cuda and logits.dtype == torch.float32 and logits.dim() == 2
    logits = logits.contiguous()
    n, vocab = logits.shape
    lp = torch.empty(n, k, dtype=torch.float32, device=logits.device)
    ids = torch.empty(n, k, dtype=torch.int32, device=logits.device)
    with torch.cuda.device(logits.device):
        _capi.check(_capi.lib().qwen35_b200_draft_topk(logits.data_ptr(), n, vocab, k, C.c_float(temperature), lp.data_ptr(), ids.data_ptr(),
                                                       C.c_void_p(torch.cuda.current_stream(logits.device).cuda_stream)), "draft_topk")
    return lp, ids


@dataclass
class DDTree:
    token_ids: np.ndarray     # int32 [1 + n], slot 0 = root (-1 until the caller fills in the root token)
    depths: np.ndarray        # int32 [1 + n]
    parents: np.ndarray       # int32 [1 + n], parents[i] < i, -1 for the root
    visibility: np.ndarray    # uint8 [1 + n, 1 + n], ancestor-or-self

    @property
    def n_nodes(self):
        return len(self.parents) - 1

    def child_maps(self):
        maps = [dict() for _ in range(len(self.parents))]
        for i in range(1, len(self.parents)):
            maps[self.parents[i]].setdefault(int(self.token_ids[i]), i)
        return maps


def build_ddtree(top_log_probs, top_token_ids, budget: int, chain_seed: bool = True) -> DDTree:
    """top_log_probs / top_token_ids: [depth_max, k] (numpy or CPU tensors)."""
    lp = np.ascontiguousarray(np.asarray(top_log_probs, dtype=np.float32))
    ids = np.ascontiguousarray(np.asarray(top_token_ids, dtype=np.int32))
    L, k = lp.shape
    tok = np.zeros(budget + 1, np.int32); dep = np.zeros(budget + 1, np.int32); par = np.zeros(budget + 1, np.int32)
    vis = np.zeros((budget + 1) * (budget + 1), np.uint8)
    n = _capi.lib().qwen35_b200_build_ddtree(lp.ctypes.data, ids.ctypes.data, L, k, budget, int(chain_seed), tok.ctypes.data, dep.ctypes.data,
                                             par.ctypes.data, vis.ctypes.data)
    if n < 0:
        raise _capi.Qwen35Error("build_ddtree: " + _capi.lib().qwen35_b200_last_error().decode())
    N = n + 1
    return DDTree(tok[:N].copy(), dep[:N].copy(), par[:N].copy(), vis[:N * N].reshape(N, N).copy())
