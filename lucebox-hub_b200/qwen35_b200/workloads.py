"""Synthetic workloads of the benchmark sections (prefill sweep, 27B-class tree verify, DFlash draft forward, NVFP4 decode,
batched decode), each timed with CUDA events and returned as a dict for the bench line.  bench.py runs them at their full
sizes; the command line of this module runs ONE of them alone at a reduced size, which is what a profiler capture needs
(few launches, a few GB on the device):

  python -m qwen35_b200.workloads tree_verify --layers 4 --iters 1
  python -m qwen35_b200.workloads draft_forward --iters 1
  python -m qwen35_b200.workloads prefill --lengths 512 --iters 1 [--nvfp4]
  python -m qwen35_b200.workloads decode --prompt 64 --gen 8
  python -m qwen35_b200.workloads decode_stages            (per-stage time table of the decode megakernel)
  python -m qwen35_b200.workloads batched --batch 64 --ctx 256 --gen 4 --kernel-table
"""
from __future__ import annotations

import json
import os
import sys

import torch

FALLBACK_HBM_GBS = 6650.0
_PEAKS = os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "..", "MEASURED_PEAKS.json")


def measured_peak():
    try:
        with open(_PEAKS) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def measured_tensor_peak() -> float:
    try:
        with open(_PEAKS) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return 1590.0


def prefill_flops(S: int) -> float:
    """Algorithmic FLOPs of one prompt: projections 2 x 498.1 M per token, causal attention 24 576 x S per
    token (6 layers x 8 heads x 4 x 256 x S/2), chunk-64 gated delta rule 47.2 M per token, one LM head."""
    return S * (2 * 498_113_344 + 24_576 * S + 47.2e6) + 2 * 254_279_680


def prefill_sweep(weights_gpu, dev, lengths, nvfp4=False, iters=5):
    """Prefill sweep configuration: batched prefill at each prompt length (ids seed 7+S): 3 warm-up runs, `iters` timed with
    CUDA events, best time reported with its share of the measured dense bf16 peak.  nvfp4=True: the fused projection and
    gate/up GEMMs and the LM head on NVFP4 operands (the flops counted stay the algorithm's)."""
    from qwen35_b200.config import QWEN35_0P8B as D
    from qwen35_b200.model import Decoder
    from qwen35_b200.weights import make_token_ids
    dec = Decoder(weights=weights_gpu, max_seq_len=max(lengths), device=dev, prefill_nvfp4=nvfp4)
    out = []
    for S in lengths:
        ids = make_token_ids(S, 7 + S, D.vocab).to(dev)
        times = []
        for i in range(3 + iters):
            dec.reset()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            dec.prefill_tokens(ids)
            e1.record()
            torch.cuda.synchronize(dev)
            if i >= 3:
                times.append(e0.elapsed_time(e1))
        dec.check_status()
        ms = min(times)
        tf = prefill_flops(S) / (ms * 1e-3) / 1e12
        out.append({"S": S, "ms": ms, "tok_s": S / (ms * 1e-3), "tflops": tf, "tensor_frac": tf / measured_tensor_peak()})
    return out


def tree_verify_bench(dev, n_nodes=33, ctx=4096, iters=5, kv_type="bf16", n_layers=0):
    """Tree-verify configuration: 27B-class dims, Q4_K weights generated directly as random super-blocks (dequantised
    sigma ~0.02), a 4096-token context of random cache contents, one 33-node tree (seeded random parents, depth <= 8):
    milliseconds per verify + accept walk + commit, timed with CUDA events."""
    from qwen35_b200.tree_verify import QWEN35_27B as T, TreeTarget, make_random_tree_weights, random_tree
    if n_layers:                      # a shallow model of the same widths: small enough for a multi-pass ncu capture
        import dataclasses
        T = dataclasses.replace(T, n_layers=n_layers)
    w = make_random_tree_weights(T, 11, device=dev)
    tt = TreeTarget(T, w, max_ctx=ctx + 128, device=dev, kv_type=kv_type)
    g = torch.Generator(device=dev).manual_seed(11)
    if kv_type in ("q8_0", "q4_0"):  # random quantised rows: f16 d = 1/127 (bytes 0x08, 0x20) or 1/8 (0x00, 0x30), codes uniform
        for c in (tt.k_cache, tt.v_cache):
            blocks = c.view(-1, 34 if kv_type == "q8_0" else 18)
            blocks.copy_(torch.randint(0, 256, blocks.shape, device=dev, generator=g, dtype=torch.uint8))
            blocks[:, 0] = 0x08 if kv_type == "q8_0" else 0x00
            blocks[:, 1] = 0x20 if kv_type == "q8_0" else 0x30
    else:
        tt.k_cache.copy_(torch.randn(tt.k_cache.shape, device=dev, generator=g).to(tt.k_cache.dtype))
        tt.v_cache.copy_(torch.randn(tt.v_cache.shape, device=dev, generator=g).to(tt.v_cache.dtype))
    tt.ssm_state.copy_(0.01 * torch.randn(tt.ssm_state.shape, device=dev, generator=g))
    tt.conv_state.copy_(0.1 * torch.randn(tt.conv_state.shape, device=dev, generator=g))
    parents = torch.tensor(random_tree(n_nodes, 8, 11), dtype=torch.int32, device=dev)
    tokens = torch.randint(0, T.vocab, (n_nodes,), dtype=torch.int32, device=dev, generator=g)
    times, acc = [], 0
    lib = tt._lib
    l0 = lib.qwen35_b200_launch_count()
    for i in range(3 + iters):
        tt.past = ctx
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        tt.verify(tokens, parents)
        tt.accept()
        acc = tt.commit()
        e1.record()
        torch.cuda.synchronize(dev)
        if i >= 3:
            times.append(e0.elapsed_time(e1))
    tt.check_status()
    launches = (lib.qwen35_b200_launch_count() - l0) // (3 + iters)
    ms = min(times)
    w_bytes = (24_352_522_240 + 1_271_398_400) * 0.5625
    kv_bytes = T.n_fa * T.kv_heads * (ctx + n_nodes) * {"bf16": T.head_dim * 2, "f16": T.head_dim * 2, "q8_0": T.head_dim // 32 * 34, "q4_0": T.head_dim // 32 * 18}[kv_type] * 2
    st_bytes = T.n_dn * n_nodes * T.dn_v_heads * T.dn_dim * T.dn_dim * 2
    alg = w_bytes + kv_bytes + st_bytes
    flops = 2 * (24_352_522_240 + 1_271_398_400) * n_nodes
    return {"workload": "tree verify: 27B-class dims (64 layers, hidden 5120), Q4_K weights, %s K/V cache, %d-token context, %d-node tree" % (kv_type, ctx, n_nodes),
            "ms_per_verify_commit": ms, "accepted": acc, "launches_per_pass": int(launches), "algorithmic_bytes": alg, "hbm_gbs": alg / (ms * 1e-3) / 1e9,
            "roofline_frac": alg / (ms * 1e-3) / 1e9 / measured_peak()[0], "tflops": flops / (ms * 1e-3) / 1e12}


def nvfp4_decode_bench(weights_gpu, dev, ids, n_gen, iters=3):
    """the same architecture with NVFP4 weights (E2M1, 16-element blocks, E4M3 block scales, fp32 tensor
    scale for the LM head; the reference pack layouts, packed by this library's own packers), bs=1, prompt 520, 128 greedy
    tokens in one launch of the NVFP4 instantiation of the decode megakernel.  Prefill runs on the BF16 weights, as the
    reference's prefill_bf16_nvfp4_lm does for the layer body."""
    from qwen35_b200.model import Decoder
    dec = Decoder(weights=weights_gpu, backend="nvfp4", max_seq_len=2048, device=dev)
    first = dec.prefill_tokens(ids)
    snap = [t.clone() for t in (dec._fa_k_cache, dec._fa_v_cache, dec._dn_states, dec._conv_bufs)]
    pos = dec._position
    times = []
    for i in range(2 + iters):
        for dst, src in zip((dec._fa_k_cache, dec._fa_v_cache, dec._dn_states, dec._conv_bufs), snap):
            dst.copy_(src)
        dec._position = pos
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        dec.step_many(first, n_gen)
        e1.record()
        torch.cuda.synchronize(dev)
        if i >= 2:
            times.append(e0.elapsed_time(e1))
    dec.check_status()
    ms = min(times)
    lc = pos + n_gen / 2.0
    alg_per_tok = 751_304_704 * 0.5625 + 1_088_320 * 2 + 2048 + 37_748_736 + 3_538_944 + 12_288 * (lc + 1)
    gbs = alg_per_tok * n_gen / (ms * 1e-3) / 1e9
    return {"workload": "NVFP4 weights, bs=1, pp520 + tg128 greedy, one launch for the 128 tokens", "tg128_tok_s": n_gen / (ms * 1e-3),
            "ms_per_token": ms / n_gen, "algorithmic_bytes_per_token": alg_per_tok, "hbm_gbs": gbs, "roofline_frac": gbs / measured_peak()[0],
            "vs_bf16_note": "same latency chain as the BF16 kernel: the stage hand-offs, not the bytes, bound both"}


def draft_forward_bench(dev, ctx=2048, iters=8):
    """Draft side of the speculative loop: the 5-layer DFlash draft at the reference's widths (hidden 5120, 32 / 8 heads of
    128, FFN 17408), bf16 random-init weights, a 2048-position feature window (the reference's cap) and 16 noise rows:
    milliseconds per forward with CUDA events.  Bytes: all draft weights once + the feature window; flops: 2 x weights x
    rows they multiply."""
    from qwen35_b200.dflash_draft import DFLASH_27B as D, DraftModel, make_random_draft_weights
    w = make_random_draft_weights(D, 5, device=dev)
    m = DraftModel(D, w, max_ctx=ctx, device=dev)
    g = torch.Generator(device=dev).manual_seed(5)
    noise = torch.randn(D.q_len, D.hidden, device=dev, generator=g).bfloat16()
    thc = torch.randn(ctx, D.n_target_layers * D.hidden, device=dev, generator=g).bfloat16()
    lib = m._lib
    times = []
    l0 = lib.qwen35_b200_launch_count()
    for i in range(3 + iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        m.forward(noise, thc)
        e1.record()
        torch.cuda.synchronize(dev)
        if i >= 3:
            times.append(e0.elapsed_time(e1))
    m.check_status()
    launches = (lib.qwen35_b200_launch_count() - l0) // (3 + iters)
    ms = min(times)
    T = ctx + D.q_len
    fc_p = D.hidden * D.n_target_layers * D.hidden
    per_layer_q = D.q_dim * D.hidden * 2 + 3 * D.inter * D.hidden            # wq, wo, gate, up, down: 16 rows each
    per_layer_kv = 2 * D.kv_dim * D.hidden                                    # wkv: all T rows
    alg = 2.0 * (fc_p + D.n_layers * (per_layer_q + per_layer_kv)) + 2.0 * ctx * D.n_target_layers * D.hidden
    flops = 2.0 * (fc_p * ctx + D.n_layers * (per_layer_q * D.q_len + per_layer_kv * T)) + D.n_layers * 4.0 * D.q_len * D.n_heads * D.head_dim * T
    return {"workload": "DFlash draft forward: 5 layers, hidden 5120, bf16, %d-position feature window + 16 noise rows" % ctx,
            "ms_per_forward": ms, "launches_per_forward": int(launches), "algorithmic_bytes": alg, "hbm_gbs": alg / (ms * 1e-3) / 1e9,
            "hbm_frac": alg / (ms * 1e-3) / 1e9 / measured_peak()[0], "tflops": flops / (ms * 1e-3) / 1e12}


def batched_decode_bench(weights_gpu, dev, rank, n_seq, ctx, n_steps, kernel_table=False, groups=1, graph=True):
    """Batched-decode configuration: `n_seq` independent sequences per GPU, `ctx`-token contexts prefilled by the library's own
    prefill, `n_steps` greedy steps.  Returns (tok/s on this rank, ms per step, algorithmic bytes per step)."""
    from qwen35_b200.config import QWEN35_0P8B as D
    from qwen35_b200.model import BatchedDecoder
    from qwen35_b200.sharding import sequence_seed
    from qwen35_b200.weights import make_token_ids
    bd = BatchedDecoder(weights_gpu, batch=n_seq, max_ctx=ctx + n_steps + 64, device=dev, groups=groups)
    for sq in range(n_seq):
        bd.prefill(sq, make_token_ids(ctx, sequence_seed(0, rank, sq), D.vocab).to(dev))
    snap = [t.clone() for t in (bd.dn_states, bd.conv_bufs, bd.positions, bd.tokens)]
    for _ in range(3):
        bd.step(graph=graph)
    for dst, src in zip((bd.dn_states, bd.conv_bufs, bd.positions, bd.tokens), snap):
        dst.copy_(src)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n_steps):
        bd.step(graph=graph)
    e1.record()
    torch.cuda.synchronize(dev)
    bd.check_status()
    if kernel_table:
        # device time per kernel of ONE step (torch.profiler / CUPTI), printed to stderr for profiles/
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            bd.step(graph=True)
            torch.cuda.synchronize(dev)
        print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=20, max_name_column_width=60), file=sys.stderr)
    ms = e0.elapsed_time(e1)
    mid = ctx + n_steps // 2
    bytes_step = 2 * (498_113_344 + 254_279_680) + n_seq * (2 * 18 * 16 * 128 * 128 * 4 + 2 * 18 * 6144 * 4 * 4 + 12288 * (mid + 2))
    del bd
    torch.cuda.empty_cache()
    return n_seq * n_steps / (ms * 1e-3), ms / n_steps, bytes_step




def decode_case(dev, prompt=64, gen=8, backend="bf16"):
    """One prefill and one launch of the decode megakernel for `gen` tokens (a profiler-sized case of the headline path)."""
    from qwen35_b200.config import QWEN35_0P8B as D
    from qwen35_b200.model import Decoder
    from qwen35_b200.weights import make_random_weights, make_token_ids, weights_to
    dec = Decoder(weights=weights_to(make_random_weights(1234, D), dev), backend=backend, max_seq_len=prompt + gen + 8, device=dev)
    first = dec.prefill_tokens(make_token_ids(prompt, 7, D.vocab).to(dev))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    toks = dec.step_many(first, gen)
    e1.record()
    torch.cuda.synchronize(dev)
    dec.check_status()
    return {"prompt": prompt, "gen": gen, "backend": backend, "ms_per_token": e0.elapsed_time(e1) / gen, "tokens": toks.tolist()[:8]}


def decode_stage_table(dev, ctx=520, gen=16, backend="bf16"):
    """Per-stage time table of the bs=1 decode megakernel: the kernel records a clock64 stamp per CTA, layer and hand-off
    (dbg_time of the decode entry point); reported are medians over the 148 CTAs and over the layers of a kind, in
    microseconds at the 1965 MHz the kernel runs at, for the last of `gen` tokens decoded from a `ctx`-token position.
    'X.in' = the stage's input vector has arrived, 'X.pub' = the CTA has published its part of the stage's output."""
    import numpy as np
    from qwen35_b200.config import QWEN35_0P8B as D
    from qwen35_b200.model import Decoder
    from qwen35_b200.weights import make_random_weights, weights_to
    dec = Decoder(weights=weights_to(make_random_weights(1234, D), dev), max_seq_len=2048, device=dev, backend=backend)
    dec.reset(); dec._position = ctx
    for _ in range(2):
        dec.step_many(5, gen)
    dec.reset(); dec._position = ctx
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(); dec.step_many(5, 128); e1.record(); torch.cuda.synchronize(dev)
    us_per_token = e0.elapsed_time(e1) * 1e3 / 128
    dec.reset(); dec._position = ctx
    tl = torch.zeros(148, 25, 12, dtype=torch.int64, device=dev)
    dec.step_many(5, gen, dbg_time=tl, dbg_time_cta=-2)
    torch.cuda.synchronize(dev)
    dec.check_status()
    t = tl.cpu().numpy().astype(np.float64) / 1965.0
    names = ["start", "A.in", "A.pub", "B.pub", "C.in", "C.pub", "D.in", "D.pub", "E.in", "E.pub"]
    out = {"us_per_token_untimed_run": us_per_token, "context": ctx, "weights": backend}
    for typ, tn in ((0, "deltanet"), (1, "attention")):
        rows = [l for l in range(4, 24) if D.layer_types[l] == typ]
        seg = {}
        for a_, b_ in zip(range(9), range(1, 10)):
            d = t[:, rows, b_] - t[:, rows, a_]
            seg[f"{names[a_]}->{names[b_]}"] = round(float(np.median(d)), 2)
        seg["layer"] = round(float(np.median(t[:, rows, 9] - t[:, rows, 0])), 2)
        out[tn] = seg
    out["lm_head"] = round(float(np.median(t[:, 24, 3] - t[:, 24, 0])), 2)
    return out


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("case", choices=["tree_verify", "draft_forward", "prefill", "decode", "decode_stages", "batched"])
    ap.add_argument("--iters", type=int, default=1)
    ap.add_argument("--layers", type=int, default=4, help="tree_verify: layers of the 27B-width model (64 = the bench's)")
    ap.add_argument("--ctx", type=int, default=256)
    ap.add_argument("--lengths", default="512")
    ap.add_argument("--nvfp4", action="store_true")
    ap.add_argument("--prompt", type=int, default=64)
    ap.add_argument("--gen", type=int, default=8)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--kernel-table", action="store_true", help="batched: print per-kernel device times of one step to stderr")
    args = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("needs a CUDA device (there is no CPU fallback)")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if args.case == "tree_verify":
        out = tree_verify_bench(dev, ctx=args.ctx, iters=args.iters, n_layers=args.layers)
    elif args.case == "draft_forward":
        out = draft_forward_bench(dev, ctx=args.ctx, iters=args.iters)
    elif args.case == "decode_stages":
        out = decode_stage_table(dev, ctx=args.ctx if args.ctx != 256 else 520, backend="nvfp4" if args.nvfp4 else "bf16")
    elif args.case == "decode":
        out = decode_case(dev, args.prompt, args.gen, "nvfp4" if args.nvfp4 else "bf16")
    else:
        from qwen35_b200.config import QWEN35_0P8B as D
        from qwen35_b200.weights import make_random_weights, weights_to
        wg = weights_to(make_random_weights(1234, D), dev)
        if args.case == "prefill":
            out = prefill_sweep(wg, dev, [int(x) for x in args.lengths.split(",")], nvfp4=args.nvfp4, iters=args.iters)
        else:
            tok_s, ms, nbytes = batched_decode_bench(wg, dev, 0, args.batch, args.ctx, args.gen, kernel_table=args.kernel_table)
            out = {"tok_s": tok_s, "ms_per_step": ms, "algorithmic_bytes_per_step": nbytes}
    print(json.dumps({args.case: out}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
