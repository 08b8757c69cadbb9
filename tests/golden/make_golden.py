"""Generate the golden fixtures in this directory from the installed `transformers`.

The reference's ground truth for its Qwen3.5 kernels is HuggingFace eager PyTorch with the
pure-torch DeltaNet functions (models/qwen35_0p8b/final_bench.py:241-304).  This script
builds `Qwen3_5ForCausalLM` (transformers 5.5.0) on CPU with eager attention and the torch
DeltaNet path, loads the seeded random-init weights of `qwen35_b200.weights`, runs a prompt
prefill followed by greedy decode, and stores tokens, logits and final states.

Two variants are written per configuration:
  *_hf.npz   the unmodified library.  Its cache stores the DeltaNet state in the dtype of
             the conv state, i.e. rounds it to bf16 after every call.
  *_f32.npz  the same run with `LinearAttentionLayer.lazy_initialization` patched so the
             state buffer keeps f32 -- what the reference kernels do (model.py:538,
             kernel.cu:684-695) and what the CUDA path is compared against.

Run from the repository root:  python tests/golden/make_golden.py [tiny|full|all]
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "lucebox-hub_b200"))

from qwen35_b200.config import QWEN35_0P8B, TINY  # noqa: E402
from qwen35_b200.weights import make_random_weights, make_token_ids  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))

sys.path.insert(0, ROOT)
from oracle.hf_reference import build_hf, greedy, patch_cache_f32  # noqa: E402


def run(model, ids, n_new):
    toks, logits, pkv, _, _ = greedy(model, ids, n_new)
    return toks, logits, pkv


def states(pkv, d):
    dn, conv, kc, vc = [], [], [], []
    for lt, layer in zip(d.layer_types, pkv.layers):
        if lt == 0:
            dn.append(layer.recurrent_states[0].float())
            conv.append(layer.conv_states[0].float())
        else:
            kc.append(layer.keys[0].float())
            vc.append(layer.values[0].float())
    return torch.stack(dn), torch.stack(conv), torch.stack(kc), torch.stack(vc)


def make(name, d, seed_w, seed_ids, n_prompt, n_new, full_logits):
    w = make_random_weights(seed_w, d)
    ids = make_token_ids(n_prompt, seed_ids, d.vocab)
    model = build_hf(w, d)
    for variant in ("hf", "f32"):
        undo = patch_cache_f32() if variant == "f32" else (lambda: None)
        toks, logits, pkv = run(model, ids, n_new)
        undo()
        dn, conv, kc, vc = states(pkv, d)
        top = torch.topk(logits, 8, dim=-1)
        rec = dict(seed_weights=seed_w, seed_ids=seed_ids, prompt_ids=ids.numpy(),
                   tokens=np.array(toks, dtype=np.int32),
                   top_vals=top.values.numpy(), top_idx=top.indices.numpy().astype(np.int32))
        if full_logits:
            rec.update(logits=logits.numpy(), dn_state=dn.numpy(), conv_state=conv.numpy(),
                       k_cache=kc.numpy(), v_cache=vc.numpy())
        else:
            # samples only: every 97th logit of every step, a few state rows, the newest K/V rows
            rec.update(logit_stride=97, logits_sampled=logits[:, ::97].numpy(),
                       dn_state_l0=dn[0, :, ::16, ::16].numpy(), dn_state_last=dn[-1, :, ::16, ::16].numpy(),
                       dn_state_norms=dn.flatten(2).norm(dim=-1).numpy(),
                       conv_state_sampled=conv[:, ::64].numpy(),
                       k_last=kc[:, :, -1].numpy(), v_last=vc[:, :, -1].numpy())
        path = os.path.join(HERE, f"{name}_{variant}.npz")
        np.savez_compressed(path, **rec)
        print(path, os.path.getsize(path), "bytes; tokens[:8] =", toks[:8])


if __name__ == "__main__":
    which = sys.argv[1] if len(sys.argv) > 1 else "all"
    if which in ("tiny", "all"):
        make("tiny_p70_g12", TINY, 1234, 7, 70, 12, True)
        make("tiny_p3_g6", TINY, 99, 5, 3, 6, True)       # prompt shorter than the conv window
    if which in ("full", "all"):
        make("qwen35_0p8b_p520_g128", QWEN35_0P8B, 1234, 7, 520, 128, False)
