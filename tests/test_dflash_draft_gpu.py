"""GPU parity of the DFlash draft forward (qwen35_b200_draft_forward through the C ABI) against the CPU oracle at reduced
widths, same seeded inputs.  Floating point: every module output is a bf16 rounding of an f32 sum whose order differs
between GPU tensor cores and the CPU, and the kernel rounds softmax probabilities to bf16; the tolerance is
|diff| <= 2^-6 * |ref| + 2^-6 per element of the final hidden state (about two bf16 steps), stated in the assertions."""
import pytest
import torch

pytestmark = pytest.mark.gpu

REL, ABS = 2.0 ** -6, 2.0 ** -6


def _dims(**kw):
    from qwen35_b200.dflash_draft import DraftDims
    base = dict(hidden=512, n_layers=2, n_heads=8, n_kv_heads=2, inter=1024)
    base.update(kw)
    return DraftDims(**base)


def _inputs(D, ctx, seed):
    g = torch.Generator().manual_seed(seed)
    noise = torch.randn(D.q_len, D.hidden, generator=g).bfloat16()
    thc = torch.randn(ctx, D.n_target_layers * D.hidden, generator=g).bfloat16() if ctx else None
    return noise, thc


@pytest.mark.parametrize("ctx", [0, 1, 128, 200, 1000])
def test_draft_forward_matches_oracle(ctx):
    """ragged context lengths: none, one row, exactly one key chunk with the noise rows spilling into a second, ragged, many chunks"""
    from oracle.dflash_draft_oracle import draft_forward
    from qwen35_b200.dflash_draft import DraftModel, draft_weights_to, make_random_draft_weights
    D = _dims()
    w = make_random_draft_weights(D, 3)
    noise, thc = _inputs(D, ctx, 11 + ctx)
    trace = []
    ref = draft_forward(D, w, noise, thc, trace=trace).float()
    m = DraftModel(D, draft_weights_to(w, "cuda"), max_ctx=1024)
    got = m.forward(noise.cuda(), thc.cuda() if ctx else None).float().cpu()
    m.check_status()
    diff = (got - ref).abs()
    print(f"ctx {ctx}: max |diff| {float(diff.max()):.4f}, mean {float(diff.mean()):.5f}, |ref| max {float(ref.abs().max()):.3f}, "
          f"{float((got != ref).float().mean()):.2%} elements differ")
    assert bool((diff <= REL * ref.abs() + ABS).all())
    assert float(diff.mean()) <= 2e-3


def test_draft_forward_is_deterministic_and_context_matters():
    from qwen35_b200.dflash_draft import DraftModel, draft_weights_to, make_random_draft_weights
    D = _dims()
    m = DraftModel(D, draft_weights_to(make_random_draft_weights(D, 5), "cuda"), max_ctx=512)
    noise, thc = _inputs(D, 300, 2)
    a = m.forward(noise.cuda(), thc.cuda())
    b = m.forward(noise.cuda(), thc.cuda())
    assert torch.equal(a, b)
    thc2 = thc.clone(); thc2[7] += 1.0
    c = m.forward(noise.cuda(), thc2.cuda())
    assert not torch.equal(a, c)                     # non-causal: every query sees every context row
    with pytest.raises(ValueError):
        m.forward(noise.cuda(), torch.zeros(513, D.n_target_layers * D.hidden, dtype=torch.bfloat16, device="cuda"))


@pytest.mark.parametrize("q4k", [False, True])
def test_draft_logits_through_the_target_head(q4k):
    """the draft has no head of its own: logits come from the target's LM head, dense bf16 or Q4_K super-blocks"""
    from oracle.dflash_draft_oracle import draft_forward
    from oracle.tree_verify_oracle import q4k_gemm_operand
    from qwen35_b200.dflash_draft import DraftModel, draft_weights_to, make_random_draft_weights
    from qwen35_b200.tree_verify import random_q4k
    D = _dims()
    vocab = 1280
    w = make_random_draft_weights(D, 9)
    noise, thc = _inputs(D, 96, 4)
    if q4k:
        blocks = random_q4k(vocab, D.hidden, 21, sigma=0.05)
        head_cpu = torch.from_numpy(q4k_gemm_operand(blocks.numpy().reshape(-1, 144))).reshape(vocab, D.hidden)
        head_gpu = blocks.cuda()
    else:
        head_cpu = (torch.randn(vocab, D.hidden, generator=torch.Generator().manual_seed(1)) * 0.05).bfloat16()
        head_gpu = head_cpu.cuda()
    ref_h, ref_l = draft_forward(D, w, noise, thc, lm_head=head_cpu)
    m = DraftModel(D, draft_weights_to(w, "cuda"), max_ctx=128, lm_head=head_gpu, lm_head_q4k=q4k, vocab=vocab)
    got_h, got_l = m.forward(noise.cuda(), thc.cuda())
    m.check_status()
    # logits of the GPU's own hidden state against the same head on the CPU: isolates the head GEMM from upstream rounding
    own = (got_h.float().cpu() @ head_cpu.float().t())
    d = (got_l.float().cpu() - own).abs()
    assert bool((d <= 2.0 ** -7 * own.abs() + 2e-3).all())
    dl = (got_l.float().cpu() - ref_l.float()).abs()
    print(f"q4k={q4k}: max |dlogit| vs oracle {float(dl.max()):.4f}")
    assert float(dl.max()) <= 0.25
