"""CPU: best-first draft tree (host code of the C library) against the Python restatement and against the properties
the algorithm guarantees."""
import numpy as np
import pytest

from oracle.ddtree_oracle import build_ddtree as oracle_build
from oracle.ddtree_oracle import draft_topk as oracle_topk


def _lists(L, K, seed, vocab=500):
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((L, vocab)).astype(np.float32) * 3
    return oracle_topk(logits, K)


@pytest.mark.parametrize("L,K,budget,chain", [(8, 4, 32, True), (8, 4, 32, False), (3, 2, 40, True), (5, 1, 10, True), (6, 8, 5, True),
                                              (6, 3, 0, True), (1, 4, 3, False)])
def test_build_ddtree_matches_restatement_and_invariants(L, K, budget, chain):
    from qwen35_b200.ddtree import build_ddtree
    lp, ids = _lists(L, K, seed=L * 100 + K)
    t = build_ddtree(lp, ids, budget, chain_seed=chain)
    tok, dep, par, vis = oracle_build(lp, ids, budget, chain)
    assert np.array_equal(t.token_ids, tok) and np.array_equal(t.depths, dep) and np.array_equal(t.parents, par) and np.array_equal(t.visibility, vis)
    n = t.n_nodes
    assert n <= budget and (n == budget or n == sum(K ** d for d in range(1, L + 1)) or K == 1)
    assert t.parents[0] == -1 and all(0 <= t.parents[i] < i for i in range(1, n + 1))
    assert all(t.depths[i] == t.depths[t.parents[i]] + 1 for i in range(1, n + 1)) and (n == 0 or t.depths.max() <= L)
    # siblings carry distinct tokens (they are distinct ranks of one top-K list), so the walk is unambiguous
    for m in t.child_maps():
        assert len(m) == len(set(m))
    # a node's log-probability is the sum along its path; nodes enter in non-increasing order of it once the chain is in
    def logw(i):
        s = 0.0
        while i > 0:
            d = t.depths[i]
            r = int(np.where(ids[d - 1] == t.token_ids[i])[0][0])
            s += float(lp[d - 1, r]); i = t.parents[i]
        return s
    start = (min(L, budget) + 1) if chain else 1
    ws = [logw(i) for i in range(start, n + 1)]
    assert all(ws[i] >= ws[i + 1] - 1e-4 for i in range(len(ws) - 1))
    # visibility is ancestor-or-self
    for i in range(n + 1):
        anc, a = set(), i
        while a >= 0:
            anc.add(a); a = t.parents[a]
        assert set(np.nonzero(t.visibility[i])[0].tolist()) == anc


def test_build_ddtree_rejects_bad_arguments():
    from qwen35_b200 import _capi
    assert _capi.lib().qwen35_b200_build_ddtree(None, None, 4, 2, 8, 1, None, None, None, None) == -1
