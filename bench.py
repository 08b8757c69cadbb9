#!/usr/bin/env python
"""Benchmark of the Qwen3.5-0.8B hybrid forward path on B200 (one JSON line on stdout).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: Qwen3.5-0.8B-architecture, seeded random-init BF16 weights, batch 1, a 520-token
uniform-random prompt, then 128 greedy decode tokens (the reference's pp520 / tg128 benchmark,
models/qwen35_0p8b/final_bench.py:158-238, with synthetic weights and ids).  One "step" is one
tg128 run: the post-prefill state is restored on the device, then 128 tokens are decoded.
  value  decode tok/s over all ranks, tokens and state resident in HBM (one launch per step)
  e2e    the same through Decoder.step(), one launch + one device->host read per token
Multi-GPU: one process per GPU (torchrun), weights replicated, one independent sequence per
rank, no collective inside the timed region ("weak" scaling); NCCL only carries the barrier and
the max-over-ranks of the elapsed time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "lucebox-hub_b200"))

import torch  # noqa: E402

from qwen35_b200.workloads import (batched_decode_bench, draft_forward_bench, measured_peak, measured_tensor_peak,  # noqa: E402
                                   nvfp4_decode_bench, prefill_flops, prefill_sweep, tree_verify_bench)

PROMPT = 520
GEN = 128


def workload_config(world: int) -> dict:
    return {"workload": "qwen35-0.8b-arch random-init bf16, bs=1 per GPU, pp%d + tg%d greedy (the reference's headline benchmark)" % (PROMPT, GEN),
            "prompt_tokens": PROMPT, "gen_tokens": GEN, "sequences_per_gpu": 1,
            "l2": "per-token working set 1.5 GB of weights >> 126 MB L2 (no flush needed)",
            "parallelism": f"replicas x{world}, no collectives"}

BASELINE_TG128 = 711.0       # the reference's published BF16 megakernel tg128 on B200 (docs/results/qwen35_0p8b_b200.md)
BASELINE_PP520 = 40278.0


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def decode_bytes(position: int) -> int:
    """Algorithmic HBM bytes of one bs=1 BF16 decode token at context length position+1:
    all weights once, embedding row, DeltaNet state and conv state read+write, K/V read of the
    whole context + one K/V row written."""
    weights = 2 * (498_113_344 + 254_279_680)
    state = 2 * 18 * 16 * 128 * 128 * 4
    conv = 2 * 18 * 6144 * 4 * 4
    kv_row = 6 * 2 * 2 * 256 * 2
    return weights + 2048 + state + conv + kv_row * (position + 1) + kv_row


class ClockSampler:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "200", "-i", str(self.idx)],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            out, _ = self.p.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
            out, _ = self.p.communicate()
        if not out.strip():            # nothing delivered in time: one query now, the GPU has just finished the region
            try:
                out = subprocess.run(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-i", str(self.idx)],
                                     capture_output=True, text=True, timeout=20).stdout
            except (OSError, subprocess.TimeoutExpired):
                out = ""
        sm, mx, reasons = [], [], set()
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1])); mx.append(float(f[2]))
            except ValueError:
                continue
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "samples": len(sm), "reasons": sorted(reasons)}


def parity_section(dec, dev):
    """Greedy-path agreement with the committed fixture of the reference's ground truth (the transformers model on the same
    seeded weights and prompt, tests/golden/qwen35_0p8b_p520_g128_f32.npz): length of the common prefix of the free-running
    128-token path, teacher-forced arg-max agreement, and for every teacher-forced disagreement the fixture's own top-2
    margin in bf16 last places of the top logit (an exact tie is 0).  Reads the fixture only; runs no CPU model."""
    import numpy as np
    path = os.path.join(ROOT, "tests", "golden", "qwen35_0p8b_p%d_g%d_f32.npz" % (PROMPT, GEN))
    if not os.path.exists(path):
        return {"unavailable": "no fixture for pp%d + tg%d" % (PROMPT, GEN)}
    g = np.load(path)
    ids = torch.from_numpy(g["prompt_ids"]).to(dev)
    gold = g["tokens"].tolist()
    first = dec.prefill_tokens(ids)
    got = [first] + dec.step_many(first, GEN - 1).tolist()
    prefix = next((i for i, (a, b) in enumerate(zip(got, gold)) if a != b), len(gold))
    first = dec.prefill_tokens(ids)
    forced = torch.tensor(gold[:-1], dtype=torch.int32, device=dev)
    tf = [first] + dec.forced_steps(forced).tolist()
    dec.check_status()
    top = g["top_vals"].astype(np.float64)
    ulp = 2.0 ** (np.floor(np.log2(np.abs(top[:, 0]))) - 7)            # one bf16 last place of the top logit
    margin_ulps = (top[:, 0] - top[:, 1]) / ulp
    agree = np.array([a == b for a, b in zip(tf, gold)])
    bad = [{"step": int(i), "fixture_margin_ulps": float(margin_ulps[i])} for i in np.nonzero(~agree)[0]]
    clear = margin_ulps > 2.0
    return {"fixture": "transformers 5.5.0 Qwen3_5ForCausalLM, f32 DeltaNet state, weights seed %d, prompt seed %d" % (int(g["seed_weights"]), int(g["seed_ids"])),
            "free_running_prefix": int(prefix), "of": len(gold),
            "teacher_forced_agreement": float(agree.mean()),
            "teacher_forced_agreement_margin_gt_2ulp": float(agree[clear].mean()) if clear.any() else None,
            "fixture_steps_with_exact_tie": int((margin_ulps == 0).sum()), "fixture_steps_within_1_ulp": int((margin_ulps <= 1).sum()),
            "fixture_min_margin_ulps": float(margin_ulps.min()),
            "teacher_forced_disagreements": bad[:24]}


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline(weights_cpu, ids, n_decode=16, use_hf=False):
    """The reference's CPU path on the host cores: one pp520 forward + `n_decode` cached greedy
    steps.  use_hf=True runs the installed transformers model itself, else the oracle port."""
    from qwen35_b200.config import QWEN35_0P8B as D
    cores = host_cores()
    torch.set_num_threads(cores)
    if use_hf:
        from oracle.hf_reference import build_hf, greedy
        model = build_hf(weights_cpu, D)
        _, _, _, t_pp, t_tg = greedy(model, ids, n_decode + 1)
        kind = "reference"
    else:
        from oracle.qwen35_oracle import Oracle
        o = Oracle(weights_cpu, D, 2048)
        t0 = time.perf_counter()
        lg = o.prefill(ids)
        t1 = time.perf_counter()
        for _ in range(n_decode):
            lg = o.step(int(lg.argmax()))
        t_pp, t_tg = t1 - t0, time.perf_counter() - t1
        kind = "port"
    return {"value": n_decode / t_tg, "unit": "tok/s", "cores": cores, "kind": kind,
            "sample": f"pp{PROMPT} once ({PROMPT / t_pp:.1f} tok/s) + {n_decode} greedy decode steps, bf16, torch CPU",
            "pp520_tok_s": PROMPT / t_pp}


def tree_cpu_baseline(n_nodes=8, layers=2, vocab=4096):
    """CPU side of the tree-verify configuration: the path-sequential oracle at the 27B widths on a reduced model (`layers` of
    64 layers, one DeltaNet + one attention; `vocab` of 248 320 LM-head rows; an 8-node chain on an empty context),
    timed per node-layer and extrapolated to 33 nodes x 64 layers.  Reported, not a target."""
    import dataclasses
    from oracle.tree_verify_oracle import TreeOracle
    from qwen35_b200.tree_verify import QWEN35_27B, make_random_tree_weights
    cores = host_cores()
    torch.set_num_threads(cores)
    T = dataclasses.replace(QWEN35_27B, n_layers=layers, fa_period=2, vocab=vocab)
    w = make_random_tree_weights(T, 11)
    orc = TreeOracle(T, w, 64)
    tokens = list(range(1, n_nodes + 1))
    t0 = time.perf_counter()
    orc.verify(tokens, [-1] + list(range(n_nodes - 1)))
    dt = time.perf_counter() - t0
    per_node_layer = dt / (n_nodes * layers)
    return {"value": per_node_layer * 33 * 64 * 1e3, "unit": "ms per verify (extrapolated)", "cores": cores, "kind": "port",
            "sample": f"{n_nodes}-node chain through {layers} of 64 layers at 27B widths (vocab {vocab}), {dt:.1f} s measured, "
                      f"scaled by 33*64/({n_nodes}*{layers}); weights dequantised once beforehand"}


def run_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return
    from qwen35_b200.config import QWEN35_0P8B as D
    from qwen35_b200.weights import make_random_weights, make_token_ids
    w = make_random_weights(1234, D)
    ids = make_token_ids(PROMPT, 7, D.vocab)
    try:
        import transformers  # noqa: F401
        use_hf = True
    except Exception:
        use_hf = False
    n_dec = 16
    vals, pps = [], []
    base = None
    t_start = time.perf_counter()
    for i in range(args.warmup + args.steps):
        base = cpu_baseline(w, ids, n_dec, use_hf)
        if i >= args.warmup:
            vals.append(base["value"]); pps.append(base["pp520_tok_s"])
        if time.perf_counter() - t_start > 240 and vals:
            break
    v = sum(vals) / len(vals)
    base["value"] = v
    line = {"impl": "reference", "metric": "decode_tg%d_tok_s" % GEN, "value": v, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": len(vals), "warmup": args.warmup, "ms_per_step": 1e3 * n_dec / v, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": workload_config(args.gpus), "sample": "each step = one pp%d forward + a %d-token greedy decode sample on the host cores" % (PROMPT, n_dec),
            "pp520_tok_s": sum(pps) / len(pps), "cpu_baseline": base,
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def run_ours(args):
    rank, local_rank, world = dist_env()
    from qwen35_b200 import _capi
    from qwen35_b200.config import QWEN35_0P8B as D
    from qwen35_b200.model import Decoder
    from qwen35_b200.weights import make_random_weights, make_token_ids, weights_to

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (there is no CPU fallback)")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)

    w_cpu = make_random_weights(1234, D)
    wg = weights_to(w_cpu, dev)
    dec = Decoder(weights=wg, max_seq_len=2048, device=dev)
    ids_cpu = make_token_ids(PROMPT, 7 + rank, D.vocab)
    ids = ids_cpu.pin_memory().to(dev, non_blocking=True)
    lib = _capi.lib()

    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731

    # ---- prefill (pp520), timed separately ----
    pp_ms = []
    for i in range(3):
        e0, e1 = ev(), ev()
        e0.record()
        first = dec.prefill_tokens(ids)
        e1.record()
        torch.cuda.synchronize(dev)
        pp_ms.append(e0.elapsed_time(e1))
    dec.check_status()
    snap = [t.clone() for t in (dec._fa_k_cache, dec._fa_v_cache, dec._dn_states, dec._conv_bufs)]

    def restore():
        for dst, src in zip((dec._fa_k_cache, dec._fa_v_cache, dec._dn_states, dec._conv_bufs), snap):
            dst.copy_(src, non_blocking=True)
        dec._position = PROMPT

    def step_device():
        restore()
        return dec.step_many(first, GEN)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    # the sampler starts before the warm-up steps (same kernels, same load): nvidia-smi needs up to a second to deliver
    # its first line, longer than a short timed region
    sampler = ClockSampler(local_rank)
    sampler.start()
    for _ in range(max(args.warmup, 3)):
        step_device()
    barrier()
    launches0 = lib.qwen35_b200_launch_count()
    k_ev = []
    barrier()
    t0, t1 = ev(), ev()
    t0.record()
    for _ in range(args.steps):
        restore()
        a, b = ev(), ev()
        a.record()
        toks = dec.step_many(first, GEN)
        b.record()
        k_ev.append((a, b))
    t1.record()
    barrier()
    launches = lib.qwen35_b200_launch_count() - launches0
    total_ms = t0.elapsed_time(t1)
    kernel_ms = [a.elapsed_time(b) for a, b in k_ev]

    # ---- e2e: the reference's host loop, Decoder.step() with one D2H read per token ----
    e2e_steps = max(1, min(args.steps, 3))
    restore(); tok = first
    for _ in range(8):
        tok = dec.step(tok)
    barrier()
    tw0 = time.perf_counter()
    e0, e1 = ev(), ev()
    e0.record()
    for _ in range(e2e_steps):
        restore(); tok = first
        for _ in range(GEN):
            tok = dec.step(tok)
    e1.record()
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    clocks = sampler.stop()
    dec.check_status()
    parity = parity_section(dec, dev) if rank == 0 else None

    sweep = sweep_fp4 = None
    if args.prefill_sweep and rank == 0:
        sweep = prefill_sweep(wg, dev, [int(x) for x in args.prefill_sweep.split(",")])
        # the same pass with its fused projection / gate-up GEMMs and the LM head on NVFP4 operands (the reference's
        # tensor-core prompt option), at the headline prompt length and the longest of the sweep
        sweep_fp4 = prefill_sweep(wg, dev, [PROMPT, 4096], nvfp4=True, iters=3)
    # the batched section runs before the 27B-class sections: those leave the GPU hot (a 1 PFLOP/s GEMM in the draft) and
    # cost the batched step ~4 % when they ran first; the other ranks of a multi-GPU run do not wait for rank 0 either
    batched = None
    if args.batched > 0:
        b_tok_s, b_ms, b_bytes = batched_decode_bench(wg, dev, rank, args.batched, args.batched_ctx, GEN, groups=args.batched_groups, graph=bool(args.batched_graph))
        from qwen35_b200.sharding import reduce_counters
        job = reduce_counters(tokens=args.batched * GEN, elapsed_ms=b_ms * GEN, algorithmic_bytes=b_bytes * GEN, device=dev)
        b_ms = job.elapsed_ms / GEN                         # slowest rank's time per step
        b_tok_s = job.tokens_per_s / world                  # per-GPU rate of the whole job
        batched = {"workload": "batched decode: %d sequences per GPU, %d-token contexts, %d greedy steps, no collectives" % (args.batched, args.batched_ctx, GEN),
                   "value": world * b_tok_s, "unit": "tok/s", "per_gpu_tok_s": b_tok_s, "ms_per_step": b_ms,
                   "algorithmic_bytes_per_step": b_bytes, "hbm_gbs": b_bytes / (b_ms * 1e-3) / 1e9,
                   "roofline_frac": b_bytes / (b_ms * 1e-3) / 1e9 / measured_peak()[0]}
    tree = draft = nvfp4 = None
    if args.tree_verify and rank == 0:
        tree = tree_verify_bench(dev)
        tree["q8_0_kv_cache_ms"] = tree_verify_bench(dev, iters=3, kv_type="q8_0")["ms_per_verify_commit"]
        tree["q4_0_kv_cache_ms"] = tree_verify_bench(dev, iters=3, kv_type="q4_0")["ms_per_verify_commit"]
        torch.cuda.empty_cache()
        draft = draft_forward_bench(dev)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([total_ms, e2e_ms, sum(kernel_ms) / len(kernel_ms)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_ms, kern_avg = t.tolist()
        cnt = torch.tensor([launches], dtype=torch.int64, device=dev)
        dist.all_reduce(cnt)
        launches = int(cnt.item())
    else:
        kern_avg = sum(kernel_ms) / len(kernel_ms)
    if args.nvfp4 and rank == 0:          # last: its allocations must not move the sections above
        try:
            nvfp4 = nvfp4_decode_bench(wg, dev, ids, GEN)
        except Exception as exc:          # reported, never hidden: the section is additive to the bench line
            nvfp4 = {"error": repr(exc)}

    if rank == 0:
        peak, peak_kind = measured_peak()
        value = world * GEN * args.steps / (total_ms * 1e-3)
        alg_bytes = sum(decode_bytes(PROMPT + i) for i in range(GEN))
        achieved = alg_bytes / (kern_avg * 1e-3) / 1e9
        traffic = None
        try:
            with open(os.path.join(ROOT, "profiles", "decode_bf16_traffic.json")) as f:
                traffic = json.load(f)["dram_bytes_per_token"] * GEN
        except Exception:
            pass
        line = {
            "metric": "decode_tg%d_tok_s" % GEN, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": (value / BASELINE_TG128) if (world == 1 and GEN == 128 and PROMPT == 520) else None,
            "dtype": "bf16", "data": "synthetic",
            "config": workload_config(world),
            "pp520_tok_s": PROMPT / (min(pp_ms) * 1e-3), "pp520_ms": min(pp_ms),
            "pp520_vs_baseline": PROMPT / (min(pp_ms) * 1e-3) / BASELINE_PP520,
            "pp520_note": "batched prefill: tcgen05 GEMMs + chunk-64 gated delta rule + causal attention + LM head, device timed",
            "prefill_roofline": {"bound": "tensor", "achieved": prefill_flops(PROMPT) / (min(pp_ms) * 1e-3) / 1e12,
                                 "peak": measured_tensor_peak(), "unit": "TFLOP/s",
                                 "frac": prefill_flops(PROMPT) / (min(pp_ms) * 1e-3) / 1e12 / measured_tensor_peak(),
                                 "flops": prefill_flops(PROMPT)},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "traffic": traffic, "kernel": "decode_stream_kernel",
                         "algorithmic_bytes_per_launch": alg_bytes, "launch_ms": kern_avg},
            "e2e": {"value": world * GEN * e2e_steps / (e2e_ms * 1e-3), "unit": "tok/s",
                    "h2d_bytes_per_step": GEN * 4, "d2h_bytes_per_step": GEN * 4,
                    "path": "Decoder.step(): per token one launch_decode (the token id travels as a launch argument), the next token stored by the kernel into pinned host memory and read after a stream synchronisation"},
            "gpu_launches": launches, "clocks": clocks,
        }
        if parity is not None:
            line["parity"] = parity
        if sweep:
            line["prefill_sweep"] = sweep
            line["prefill_sweep_nvfp4"] = sweep_fp4
        if tree:
            line["tree_verify"] = tree
        if draft is not None:
            line["draft_forward"] = draft
        if nvfp4 is not None:
            line["nvfp4_decode"] = nvfp4
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(w_cpu, ids_cpu, 16, use_hf=False)
            if batched:
                # the CPU runs the sequences one after another, so its aggregate rate is its single-sequence rate
                batched["cpu_baseline"] = {"value": line["cpu_baseline"]["value"], "unit": "tok/s", "cores": line["cpu_baseline"]["cores"], "kind": "port",
                                           "sample": "single-sequence decode rate of the bs=1 sample (the CPU path has no batching); context 520 instead of 2048"}
            if tree:
                tree["cpu_baseline"] = tree_cpu_baseline()
        if batched:
            line["batched_decode"] = batched          # last key: the per-N aggregate stays in the tail of the line
        print(json.dumps(line))
    if world > 1:
        torch.distributed.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batched", type=int, default=64, help="sequences per GPU for the batched-decode section (0 = skip)")
    ap.add_argument("--batched-ctx", type=int, default=2048)
    ap.add_argument("--batched-groups", type=int, default=1, help="concurrent sub-batches of the batched-decode step (1 = one batch)")
    ap.add_argument("--prefill-sweep", default="128,512,1024,4096", help="prompt lengths of the prefill sweep ('' = skip)")
    ap.add_argument("--batched-graph", type=int, default=1, help="1: replay the batched step as a CUDA graph (default); 0: launch it eagerly")
    ap.add_argument("--nvfp4", type=int, default=1, help="run the NVFP4-weights decode section (0 = skip)")
    ap.add_argument("--tree-verify", type=int, default=1, help="run the 27B-class tree-verify section (0 = skip)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
