"""GPU parity tests of the BF16 decode megakernel, called through the C ABI
(libqwen35_b200.so via qwen35_b200.model.Decoder), against the CPU oracle.

What "parity" means here.  A bf16 network of this width is rounding-chaotic: one bf16 last-place
flip inside one layer changes hundreds of that layer's outputs and, 24 layers later, almost every
logit (tests/test_oracle_sensitivity.py measures it on the oracle alone).  Two correct
implementations whose f32 sums run in a different order therefore agree bit for bit on most
layer outputs but not on the end-to-end logits.  The gates are:
  * layer level, teacher forced (each GPU layer is fed the oracle's input of that layer): most
    layers bit-identical, every element within LAYER_ABS_TOL, DeltaNet state within 1e-3
    relative (the tolerance the task states), conv / K / V rows within one bf16 last place;
  * model level: logits agree with the oracle as closely as the oracle agrees with itself under
    a one-last-place perturbation, and the arg-max is identical whenever the oracle's top-2
    margin exceeds that noise;
  * exact self-consistency of the CUDA path (step vs step_many, run to run).
"""
import numpy as np
import pytest
import torch

from conftest import load_golden
from helpers import bf16_ulps, load_oracle_state

pytestmark = pytest.mark.gpu

LAYER_ABS_TOL = 2.0 ** -5        # absolute bound on any layer-output element, hidden scale is 1..4
STATE_REL_TOL = 1e-3             # DeltaNet state, relative Frobenius error
LOGIT_TOL = 2e-2                 # teacher-forced logits (computed from the GPU's own last-layer output): the task's bound
LOGIT_NOISE = 0.30               # free-running logits only: 2x the oracle's own 1-ulp sensitivity over 24 layers (0.08-0.15)


@pytest.fixture(scope="module")
def ctx(full_weights_cpu):
    from oracle.qwen35_oracle import Oracle
    from qwen35_b200.config import QWEN35_0P8B as D
    from qwen35_b200.model import Decoder
    from qwen35_b200.weights import make_token_ids, weights_to
    wg = weights_to(full_weights_cpu, "cuda")
    dec = Decoder(weights=wg, max_seq_len=2048)
    return dict(D=D, w=full_weights_cpu, dec=dec, Oracle=Oracle, ids=make_token_ids(64, 7, D.vocab))


@pytest.mark.parametrize("n_prompt", [1, 3, 40, 648])
def test_layer_parity_teacher_forced(ctx, n_prompt):
    """648 = the last context length of the benchmarked pp520 + tg128 run (21 attention chunks of 31 positions)."""
    D, dec = ctx["D"], ctx["dec"]
    ids = ctx["ids"]
    if n_prompt >= len(ids):
        from qwen35_b200.weights import make_token_ids
        ids = make_token_ids(n_prompt + 1, 7, D.vocab)
    o = ctx["Oracle"](ctx["w"], D, 2048)
    o.prefill(ids[:n_prompt])
    load_oracle_state(dec, o)
    ref_logits = o.step(int(ids[n_prompt]))
    trace = torch.stack(o.trace)
    teacher = torch.zeros(24, 1024, dtype=torch.bfloat16)
    teacher[1:] = trace[:-1]
    dbg = torch.zeros(24, 1024, dtype=torch.bfloat16, device="cuda")
    logits = torch.zeros(D.vocab, device="cuda")
    tok = dec.forced_steps(ids[n_prompt:n_prompt + 1].cuda(), logits_out=logits, dbg_hidden=dbg,
                           dbg_teacher=teacher.cuda())
    dec.check_status()
    got = dbg.cpu()
    exact_layers = int((got == trace).all(dim=1).sum())
    frac_diff = float((got != trace).float().mean())
    max_abs = float((got.float() - trace.float()).abs().max())
    print(f"n_prompt={n_prompt}: {exact_layers}/24 layers bit-identical, {frac_diff:.4%} elements differ, max abs {max_abs}")
    # measured 15-20 of 24 (which layers match moves with the order of the f32 sums; the share of differing elements does not)
    assert exact_layers >= 12
    assert frac_diff < 0.05
    assert max_abs <= LAYER_ABS_TOL
    # logits of the last layer's (GPU) output: same arg-max, small deviation
    ld = (logits.cpu() - ref_logits.float()).abs()
    print(f"n_prompt={n_prompt}: teacher-forced max |dlogit| {float(ld.max()):.4f}")
    assert float(ld.max()) <= LOGIT_TOL
    margin = torch.topk(ref_logits.float(), 2).values
    if float(margin[0] - margin[1]) > 2 * float(ld.max()):
        assert int(tok[0]) == int(ref_logits.argmax())
    # states after the step
    st, st_ref = dec._dn_states.cpu(), o.dn_states_ref_layout()
    assert float((st - st_ref).norm() / st_ref.norm()) <= STATE_REL_TOL
    cv, cv_ref = dec._conv_bufs.cpu(), o.conv_ref_layout()
    assert float((cv != cv_ref).float().mean()) < 0.01
    assert float((cv - cv_ref).abs().max()) <= 2.0 ** -5
    k_new = dec._fa_k_cache[:, :, n_prompt].cpu()
    v_new = dec._fa_v_cache[:, :, n_prompt].cpu()
    assert int(bf16_ulps(k_new, torch.stack(o.k_cache)[:, :, n_prompt]).max()) <= 4
    assert int(bf16_ulps(v_new, torch.stack(o.v_cache)[:, :, n_prompt]).max()) <= 4
    # older cache rows are untouched
    assert torch.equal(dec._fa_k_cache[:, :, :n_prompt].cpu(), torch.stack(o.k_cache)[:, :, :n_prompt])


def test_model_level_logits_and_argmax(ctx):
    """Token-serial GPU prefill of 24 tokens vs the oracle run token by token (same recurrence
    form), then the first generated token."""
    D, dec = ctx["D"], ctx["dec"]
    ids = ctx["ids"][:24]
    o = ctx["Oracle"](ctx["w"], D, 2048)
    for t in ids.tolist():
        ref = o.step(t)
    logits = torch.zeros(D.vocab, device="cuda")
    tok = dec.prefill_tokens(ids.cuda(), logits_out=logits)
    dec.check_status()
    got, ref = logits.cpu(), ref.float()
    diff = (got - ref).abs()
    corr = float(torch.corrcoef(torch.stack([got, ref]))[0, 1])
    print(f"logits: max abs diff {float(diff.max()):.4f}, mean {float(diff.mean()):.5f}, corr {corr:.6f}")
    assert float(diff.max()) <= LOGIT_NOISE
    assert corr > 0.995
    top = torch.topk(ref, 2).values
    if float(top[0] - top[1]) > 2 * float(diff.max()):
        assert tok == int(ref.argmax())
    st, st_ref = dec._dn_states.cpu(), o.dn_states_ref_layout()
    rel = float((st - st_ref).norm() / st_ref.norm())
    print("DeltaNet state relative error after 24 tokens:", rel)
    assert rel < 5e-2          # free-running: bounded by the network's rounding sensitivity, not by 1e-3


def test_golden_prompt_greedy_prefix(ctx):
    """pp520 + tg128 on the golden prompt: report how far the free-running greedy path follows
    the fixture, and require exact agreement at teacher-forced steps with a clear margin."""
    D, dec = ctx["D"], ctx["dec"]
    g = load_golden("qwen35_0p8b_p520_g128_f32")
    ids = torch.from_numpy(g["prompt_ids"]).cuda()
    first = dec.prefill_tokens(ids)
    rest = dec.step_many(first, 127).tolist()
    dec.check_status()
    got = [first] + rest
    gold = g["tokens"].tolist()
    prefix = next((i for i, (a, b) in enumerate(zip(got, gold)) if a != b), len(gold))
    print(f"free-running greedy: common prefix with the fixture {prefix}/128 tokens")
    assert all(0 <= t < D.vocab for t in got)
    # teacher forced on the fixture's tokens
    first = dec.prefill_tokens(ids)
    forced = torch.tensor(gold[:-1], dtype=torch.int32, device="cuda")
    tf = [first] + dec.forced_steps(forced).tolist()
    dec.check_status()
    margins = g["top_vals"][:, 0] - g["top_vals"][:, 1]
    agree = np.array([a == b for a, b in zip(tf, gold)])
    print(f"teacher-forced arg-max agreement {agree.mean():.3f}; on steps with margin > {LOGIT_NOISE}: "
          f"{agree[margins > LOGIT_NOISE].mean() if (margins > LOGIT_NOISE).any() else float('nan'):.3f}")
    assert agree[margins > LOGIT_NOISE].all()
    assert agree.mean() > 0.5


def test_step_equals_step_many_and_is_deterministic(ctx):
    dec = ctx["dec"]
    ids = ctx["ids"][:8].cuda()
    t0 = dec.prefill_tokens(ids)
    many = dec.step_many(t0, 12).tolist()
    t0b = dec.prefill_tokens(ids)
    assert t0b == t0
    one, tok = [], t0
    for _ in range(12):
        tok = dec.step(tok)
        one.append(tok)
    again = None
    t0c = dec.prefill_tokens(ids)
    again = dec.step_many(t0c, 12).tolist()
    dec.check_status()
    assert one == many == again


def test_argument_checks(ctx):
    from qwen35_b200._capi import Qwen35Error
    dec = ctx["dec"]
    dec.reset()
    dec._position = dec.max_seq_len
    with pytest.raises(Qwen35Error):
        dec.step(1)
    dec._position = 0
    with pytest.raises(Qwen35Error):
        dec.step(10 ** 9)
    with pytest.raises(TypeError):
        dec.prefill_tokens(torch.zeros(4, dtype=torch.int64, device="cuda"))
    dec.check_status()


def test_gpu_is_as_close_to_the_exact_evaluation_as_the_reference_order_is(ctx):
    """Two correct bf16 implementations differ where their f32 sums straddle a rounding boundary.  To show that what
    separates the CUDA path from the oracle is that and nothing else, both are compared with a third evaluation in which
    every projection is summed exactly (f64) and rounded once.  Layer level, teacher forced on the oracle's inputs, three
    decode steps at different contexts: the CUDA path must not sit further from the exact values than the
    HuggingFace-order oracle does (factor 1.5 plus a small constant for the counting noise of a handful of flips)."""
    import copy
    import oracle.qwen35_oracle as Q
    from qwen35_b200.weights import make_token_ids
    D, dec = ctx["D"], ctx["dec"]
    tot_hf = tot_gpu = 0
    per_layer_hf, per_layer_gpu = torch.zeros(24, dtype=torch.long), torch.zeros(24, dtype=torch.long)
    max_hf = max_gpu = 0.0
    for n_prompt, seed in ((5, 21), (70, 22), (200, 23)):
        ids = make_token_ids(n_prompt + 1, seed, D.vocab)
        o = ctx["Oracle"](ctx["w"], D, 2048)
        o.prefill(ids[:n_prompt])
        oe = copy.deepcopy(o)
        load_oracle_state(dec, o)
        o.step(int(ids[n_prompt]))
        trace = torch.stack(o.trace)
        teacher_rows = [None] + [trace[i][None] for i in range(23)]
        Q.EXACT_LINEAR = True
        try:
            oe.step(int(ids[n_prompt]), teacher=teacher_rows)
        finally:
            Q.EXACT_LINEAR = False
        exact = torch.stack(oe.trace)
        teacher = torch.zeros(24, 1024, dtype=torch.bfloat16)
        teacher[1:] = trace[:-1]
        dbg = torch.zeros(24, 1024, dtype=torch.bfloat16, device="cuda")
        dec.forced_steps(ids[n_prompt:n_prompt + 1].cuda(), dbg_hidden=dbg, dbg_teacher=teacher.cuda())
        dec.check_status()
        got = dbg.cpu()
        per_layer_hf += (trace != exact).sum(dim=1)
        per_layer_gpu += (got != exact).sum(dim=1)
        max_hf = max(max_hf, float((trace.float() - exact.float()).abs().max()))
        max_gpu = max(max_gpu, float((got.float() - exact.float()).abs().max()))
    tot_hf, tot_gpu = int(per_layer_hf.sum()), int(per_layer_gpu.sum())
    print(f"layer outputs differing from the exactly-rounded evaluation over 3 steps x 24 layers x 1024: reference-order oracle {tot_hf}, "
          f"CUDA path {tot_gpu}; max |diff| {max_hf} vs {max_gpu}")
    print("  per layer (oracle / CUDA):", list(zip(per_layer_hf.tolist(), per_layer_gpu.tolist())))
    assert tot_gpu <= 1.5 * tot_hf + 64
    assert max_gpu <= max(2 * max_hf, 2.0 ** -6)
