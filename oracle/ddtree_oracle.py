"""TEST INFRASTRUCTURE ONLY: numpy / pure-Python restatement of the draft-tree host logic of the reference's driver
(models/qwen35_27b/test/test_dflash.cpp:143-207 top-K log-probabilities, :218-390 best-first tree).  The reference
stores no expected values for it; the restatement follows its published algorithm and is checked for the properties
the algorithm guarantees (tests/test_ddtree_cpu.py).  Ties: equal values by ascending token id (top-K), equal
log-probabilities by creation order (tree) -- the reference leaves both to the heap implementation."""
import heapq

import numpy as np


def draft_topk(logits: np.ndarray, k: int, temperature: float = 1.0):
    x = logits.astype(np.float32) * np.float32(1.0 / max(1e-3, temperature))
    mx = x.max(axis=1, keepdims=True)
    log_z = mx[:, 0] + np.log(np.exp(x - mx).sum(axis=1, dtype=np.float32))
    order = np.lexsort((np.arange(x.shape[1])[None, :].repeat(x.shape[0], 0), -x), axis=1)[:, :k]      # value desc, id asc
    vals = np.take_along_axis(x, order, axis=1)
    return (vals - log_z[:, None]).astype(np.float32), order.astype(np.int32)


def build_ddtree(lp: np.ndarray, ids: np.ndarray, budget: int, chain_seed: bool = True):
    L, K = lp.shape
    tokens, depths, parents = [-1], [0], [-1]
    heap, seq = [], 0
    lp = lp.astype(np.float32)

    def push(logw, parent, depth, rank):
        nonlocal seq
        heapq.heappush(heap, (-float(np.float32(logw)), seq, parent, depth, rank)); seq += 1

    def add(parent, depth, rank):
        tokens.append(int(ids[depth - 1, rank])); depths.append(depth); parents.append(parent)
        return len(parents) - 1

    if budget > 0 and L > 0:
        if chain_seed:
            cum, prev = np.float32(0), 0
            for d in range(1, L + 1):
                if len(parents) - 1 >= budget:
                    break
                cum = np.float32(cum + lp[d - 1, 0])
                cur = add(prev, d, 0)
                if K > 1:
                    push(np.float32(np.float32(cum - lp[d - 1, 0]) + lp[d - 1, 1]), prev, d, 1)
                prev = cur
        else:
            push(lp[0, 0], 0, 1, 0)
        while heap and len(parents) - 1 < budget:
            neg, _, parent, depth, rank = heapq.heappop(heap)
            logw = np.float32(-neg)
            cur = add(parent, depth, rank)
            if rank + 1 < K:
                push(np.float32(np.float32(logw - lp[depth - 1, rank]) + lp[depth - 1, rank + 1]), parent, depth, rank + 1)
            if depth < L:
                push(np.float32(logw + lp[depth, 0]), cur, depth + 1, 0)
    N = len(parents)
    vis = np.zeros((N, N), np.uint8)
    for i in range(N):
        if i:
            vis[i, :i] = vis[parents[i], :i]
        vis[i, i] = 1
    return np.array(tokens, np.int32), np.array(depths, np.int32), np.array(parents, np.int32), vis
