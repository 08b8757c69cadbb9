"""Why end-to-end bit-exactness is not a usable gate on random-init bf16 weights: the oracle
alone, perturbed by ONE bf16 last-place flip of ONE normalised activation in layer 1, changes
hundreds of that layer's outputs and most of the final logits by far more than 2e-2."""
import torch

import oracle.qwen35_oracle as OQ
from qwen35_b200.config import QWEN35_0P8B
from qwen35_b200.weights import make_token_ids


def test_one_ulp_flip_reaches_the_logits(full_weights_cpu, monkeypatch):
    ids = make_token_ids(1, 7, QWEN35_0P8B.vocab)
    base = OQ.Oracle(full_weights_cpu, QWEN35_0P8B)
    lb = base.prefill(ids).float()
    tb = torch.stack(base.trace).float()

    orig = OQ.rmsnorm
    calls = {"n": 0}

    def flipped(x, w, eps):
        out = orig(x, w, eps)
        calls["n"] += 1
        if calls["n"] == 3:                      # input norm of layer 1
            out = out.clone()
            out[..., 5] = (out[..., 5].float() * (1 + 2 ** -8)).to(out.dtype)
        return out

    monkeypatch.setattr(OQ, "rmsnorm", flipped)
    pert = OQ.Oracle(full_weights_cpu, QWEN35_0P8B)
    lp = pert.prefill(ids).float()
    tp = torch.stack(pert.trace).float()
    changed_l1 = int((tb[1] != tp[1]).sum())
    changed_last = int((tb[-1] != tp[-1]).sum())
    max_logit = float((lb - lp).abs().max())
    print(f"layer-1 outputs changed: {changed_l1}/1024, last layer: {changed_last}/1024, max |dlogit| {max_logit}")
    assert torch.equal(tb[0], tp[0])
    assert changed_l1 > 100
    assert changed_last > 512
    assert max_logit > 2e-2
