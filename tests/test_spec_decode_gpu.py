"""The speculative loop end to end on the GPU (draft forward -> top-k -> best-first tree -> tree verify -> accept ->
commit) at reduced widths with random weights.  Greedy verification makes the loop's output the target's own greedy
continuation, whatever the draft proposes: the test decodes the same prompt one token at a time with the same target
and compares.  A token may differ only where the target's two best logits are closer than the bf16 noise of the two
evaluation orders (tree slots vs sequential slots); comparison stops there because the continuations then diverge."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LOGIT_NOISE = 3e-2


def _build(seed, budget, feat_cap=96):
    from qwen35_b200.dflash_draft import DraftDims, make_random_draft_weights
    from qwen35_b200.spec_decode import SpecDecoder
    from qwen35_b200.tree_verify import TreeDims, TreeTarget, make_random_tree_weights
    T = TreeDims(n_layers=4, hidden=512, ffn=1024, vocab=2048, q_heads=4, kv_heads=2, dn_k_heads=2, dn_v_heads=4)
    w = make_random_tree_weights(T, seed)
    wg = {"layers": [{k: v.cuda() for k, v in L.items()} for L in w["layers"]],
          "token_embd": w["token_embd"].cuda(), "output_norm": w["output_norm"].cuda(), "output_w": w["output_w"].cuda()}
    D = DraftDims(hidden=512, n_layers=2, n_heads=8, n_kv_heads=2, inter=1024, n_target_layers=2)

    def target():
        return TreeTarget(T, wg, max_ctx=512, capture_layers=(1, 3), feat_cap=feat_cap)
    dw = make_random_draft_weights(D, seed + 1, device="cuda")
    return T, wg, D, dw, target, SpecDecoder


@pytest.mark.parametrize("budget,prompt_len", [(32, 50), (6, 3), (39, 41)])
def test_spec_loop_reproduces_sequential_greedy(budget, prompt_len):
    T, wg, D, dw, target, SpecDecoder = _build(5 + budget, budget)
    rng = np.random.default_rng(budget)
    prompt = rng.integers(0, T.vocab, prompt_len)
    n_gen = 24
    sd = SpecDecoder(target(), wg, D, dw, mask_token_id=T.vocab - 1, budget=budget)
    got = sd.generate(prompt, n_gen)
    sd.target.check_status()
    assert len(got) == n_gen and all(0 <= t < T.vocab for t in got)
    assert sd.stats["committed"] >= sd.stats["steps"] >= 1                  # every round commits at least the root
    assert sd.target.past == prompt_len + sd.stats["committed"]
    # the same target, one token per verify
    ref_t = target()
    seq = SpecDecoder(ref_t, wg, D, dw, mask_token_id=T.vocab - 1, budget=1)
    tok = seq.prefill(prompt)
    ref, gaps = [tok], []
    logits = torch.zeros(1, T.vocab, dtype=torch.bfloat16, device="cuda")
    for _ in range(n_gen - 1):
        am = ref_t.verify(torch.tensor([tok], dtype=torch.int32), torch.tensor([-1], dtype=torch.int32), logits_out=logits)
        top = torch.topk(logits[0].float(), 2).values
        gaps.append(float(top[0] - top[1]))
        ref_t.commit(torch.zeros(1, dtype=torch.int32, device="cuda"), torch.stack([torch.ones((), dtype=torch.int32, device="cuda"), am[0]]).to(torch.int32))
        tok = int(am[0].item())
        ref.append(tok)
    same = 0
    for i in range(n_gen):
        if got[i] != ref[i]:
            assert i >= 1 and gaps[i - 1] <= 2 * LOGIT_NOISE, (i, got[i], ref[i], gaps[i - 1])
            break
        same += 1
    print(f"budget {budget}: {same}/{n_gen} tokens equal the sequential greedy run; rounds {sd.stats['steps']}, "
          f"committed {sd.stats['committed']}, mean tree {sd.stats['tree_nodes'] / sd.stats['steps']:.1f} nodes")
    assert same >= 2


def test_spec_loop_accepts_deep_paths_from_a_knowing_draft():
    """Several tokens per round: the proposal is replaced by the target's own greedy look-ahead (computed on a second
    target instance kept in lockstep, snapshot / restore around the look-ahead), so whole chains are accepted and
    committed.  Every emitted token must be the lockstep target's arg-max given the same prefix, or within the bf16 noise
    of it (deep tree nodes see their keys in other cache slots than a sequential run: another f32 summation order; with
    random weights the two best logits are often that close)."""
    budget, prompt_len, n_gen = 32, 20, 40
    T, wg, D, dw, target, SpecDecoder = _build(77, budget)
    prompt = np.random.default_rng(3).integers(0, T.vocab, prompt_len)
    sd = SpecDecoder(target(), wg, D, dw, mask_token_id=T.vocab - 1, budget=budget)
    look = target()
    lock = SpecDecoder(look, wg, D, dw, mask_token_id=T.vocab - 1, budget=1)
    out = [sd.prefill(prompt)]
    assert lock.prefill(prompt) == out[0]
    logits = torch.zeros(1, T.vocab, dtype=torch.bfloat16, device="cuda")
    zero = torch.zeros(1, dtype=torch.int32, device="cuda")

    def one(tok):
        am = look.verify(torch.tensor([tok], dtype=torch.int32), torch.tensor([-1], dtype=torch.int32), logits_out=logits)
        look.commit(zero, torch.stack([torch.ones((), dtype=torch.int32, device="cuda"), am[0]]).to(torch.int32))
        return int(am[0].item())

    ahead = []
    real_forward = sd.draft.forward

    def knowing_forward(noise, window):
        hidden, lg = real_forward(noise, window)              # the real kernels still run; only the proposal is replaced
        lg = torch.full_like(lg, -4.0)
        for j in range(1, D.q_len):
            lg[j, ahead[j - 1]] = 8.0
        return hidden, lg
    sd.draft.forward = knowing_forward
    near_ties = 0
    while len(out) < n_gen:
        root = sd.last_token
        snap = (look.k_cache.clone(), look.v_cache.clone(), look.ssm_state.clone(), look.conv_state.clone(), look.past)
        ahead.clear(); tok = root
        for _ in range(D.q_len - 1):
            tok = one(tok); ahead.append(tok)
        look.k_cache.copy_(snap[0]); look.v_cache.copy_(snap[1]); look.ssm_state.copy_(snap[2]); look.conv_state.copy_(snap[3]); look.past = snap[4]
        new = sd.step()
        tok = root
        for t_new in new:                                     # replay the round on the lockstep target, token by token
            am = one(tok)
            lg = logits[0].float()
            if t_new != am:
                near_ties += 1
                assert float(lg.max() - lg[t_new]) <= 2 * LOGIT_NOISE, (len(out), t_new, am)
            tok = t_new
        assert look.past == sd.target.past
        out.extend(new)
    sd.target.check_status()
    per_round = sd.stats["committed"] / sd.stats["steps"]
    print(f"knowing draft: {sd.stats['steps']} rounds for {len(out)} tokens, {per_round:.1f} committed per round, {near_ties} near-tie choices")
    assert per_round >= 2.0


def test_spec_loop_argument_checks():
    T, wg, D, dw, target, SpecDecoder = _build(1, 8)
    from qwen35_b200.tree_verify import TreeTarget
    with pytest.raises(ValueError):
        SpecDecoder(TreeTarget(T, wg, max_ctx=64), wg, D, dw, mask_token_id=0)            # no feature ring
    with pytest.raises(ValueError):
        SpecDecoder(target(), wg, D, dw, mask_token_id=0, budget=40)
    sd = SpecDecoder(target(), wg, D, dw, mask_token_id=0, budget=8)
    with pytest.raises(RuntimeError):
        sd.step()
    with pytest.raises(ValueError):
        sd.prefill([])
