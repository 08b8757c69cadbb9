"""Seed selection rule for the published weight / prompt seeds, evaluated on the CPU oracle only.

Rule (stated before looking at any GPU result): take the first (weight seed, prompt seed) pair, in the order scanned,
whose greedy pp520 + tg128 run on the CPU oracle has NO exact tie at the bf16 arg-max in any of the 128 steps and whose
smallest top-2 margin is at least 2 bf16 last places of the top logit.  If no scanned pair qualifies, keep the first pair
and publish the table: on random-init weights the top-2 margin of a 248 320-way soft-max is small by construction.

Writes tests/golden/seed_scan.json: per pair the number of exact bf16 ties, of steps within 1 and 2 last places, the
smallest margin (in logit units and in last places) and the step where it occurs.

Usage: python tests/golden/scan_seeds.py [n_pairs]
"""
import json
import os
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (ROOT, os.path.join(ROOT, "lucebox-hub_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

PAIRS = [(1234, 7), (1, 1), (2, 2), (3, 3), (5, 11), (42, 42), (100, 200), (2024, 1), (7, 1234), (31337, 5), (8, 8), (13, 21)]


def bf16_ulp(x: float) -> float:
    t = torch.tensor([x], dtype=torch.bfloat16)
    nxt = (t.view(torch.int16) + 1).view(torch.bfloat16)
    return float(nxt.float() - t.float())


def scan_pair(wseed, pseed, prompt=520, gen=128):
    from oracle.qwen35_oracle import Oracle
    from qwen35_b200.config import QWEN35_0P8B as D
    from qwen35_b200.weights import make_random_weights, make_token_ids
    w = make_random_weights(wseed, D)
    ids = make_token_ids(prompt, pseed, D.vocab)
    o = Oracle(w, D, prompt + gen)
    toks, logits = o.generate(ids, gen)
    ties = w1 = w2 = 0
    worst, worst_step, worst_ulps = 1e9, -1, 1e9
    for i, lg in enumerate(logits):
        top = torch.topk(lg.float(), 2).values
        gap = float(top[0] - top[1])
        u = gap / bf16_ulp(float(top[0]))
        ties += gap == 0.0
        w1 += u <= 1.0
        w2 += u <= 2.0
        if gap < worst:
            worst, worst_step, worst_ulps = gap, i, u
    return {"weight_seed": wseed, "prompt_seed": pseed, "exact_ties": int(ties), "within_1_ulp": int(w1), "within_2_ulp": int(w2),
            "min_margin": worst, "min_margin_ulps": worst_ulps, "min_margin_step": worst_step, "first_tokens": toks[:4]}


def main():
    n = int(sys.argv[1]) if len(sys.argv) > 1 else len(PAIRS)
    rows = []
    for ws, ps in PAIRS[:n]:
        t0 = time.time()
        r = scan_pair(ws, ps)
        r["qualifies"] = bool(r["exact_ties"] == 0 and r["min_margin_ulps"] >= 2.0)
        rows.append(r)
        print(r, f"{time.time() - t0:.0f}s", flush=True)
        with open(os.path.join(HERE, "seed_scan.json"), "w") as f:
            json.dump({"rule": "first pair with no exact bf16 tie and min top-2 margin >= 2 bf16 last places over 128 greedy steps",
                       "prompt_tokens": 520, "gen_tokens": 128, "pairs": rows,
                       "chosen": next(([x["weight_seed"], x["prompt_seed"]] for x in rows if x["qualifies"]), [PAIRS[0][0], PAIRS[0][1]])}, f, indent=1)


if __name__ == "__main__":
    main()
