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
    # a draft that knows the continuation: several tokens are accepted per round and the output stays the greedy one
    if same == n_gen:
        sd2 = SpecDecoder(target(), wg, D, dw, mask_token_id=T.vocab - 1, budget=budget)
        out2 = [sd2.prefill(prompt)]
        real_forward = sd2.draft.forward

        def knowing_forward(noise, window):
            hidden, logits = real_forward(noise, window)          # the real kernels still run; only the proposal is replaced
            logits = torch.full_like(logits, -4.0)
            for j in range(1, D.q_len):
                idx = len(out2) + j - 1
                logits[j, ref[idx] if idx < n_gen else 0] = 8.0
            return hidden, logits
        sd2.draft.forward = knowing_forward
        while len(out2) < n_gen:
            out2.extend(sd2.step())
        sd2.target.check_status()
        agree = sum(1 for a, b in zip(out2[:n_gen], ref) if a == b)
        print(f"  with a knowing draft: {sd2.stats['steps']} rounds for {n_gen} tokens, {sd2.stats['committed'] / sd2.stats['steps']:.1f} committed per round, "
              f"{agree}/{n_gen} tokens equal")
        assert sd2.stats["steps"] < sd.stats["steps"] and sd2.stats["committed"] / sd2.stats["steps"] >= 2.0
        first_diff = next((i for i in range(n_gen) if out2[i] != ref[i]), n_gen)
        assert first_diff == n_gen or gaps[first_diff - 1] <= 2 * LOGIT_NOISE


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
