"""GPU parity of batched decode (B sequences per step) against the bs=1 CPU oracle, sequence by sequence,
layer level and teacher forced, through the C ABI (qwen35_b200_decode_batched)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

LAYER_ABS_TOL = 2.0 ** -5
# share of a teacher-forced trace's elements (24 layers x 1024) that may sit one bf16 step from the oracle's: one flipped
# rounding early in a layer moves a few hundred of that layer's outputs, so the share moves in steps with the order of the
# f32 sums in the GEMMs (measured 2.7-5.7 % per sequence over the split-K and the full-K forms of the same GEMM)
FRAC_TOL = 0.08
STATE_REL_TOL = 1e-3
LOGIT_TOL = 2e-2                 # teacher-forced logits: the task's bound


def test_batched_step_matches_oracle_per_sequence(full_weights_cpu):
    from oracle.qwen35_oracle import Oracle
    from qwen35_b200.config import QWEN35_0P8B as D
    from qwen35_b200.model import BatchedDecoder
    from qwen35_b200.weights import make_token_ids, weights_to
    wg = weights_to(full_weights_cpu, "cuda")
    lens = [1, 9, 70, 130]                      # ragged contexts, one crossing a 64-position page and a chunk boundary
    B = len(lens)
    bd = BatchedDecoder(wg, batch=B, max_ctx=256)
    oracles, traces, ref_logits, nxt = [], [], [], []
    teacher = torch.zeros(24, B, 1024, dtype=torch.bfloat16)
    for b, L in enumerate(lens):
        ids = make_token_ids(L + 1, 100 + b, D.vocab)
        o = Oracle(full_weights_cpu, D, 256)
        o.prefill(ids[:L])
        bd.load_sequence(b, torch.stack(o.k_cache).cuda(), torch.stack(o.v_cache).cuda(), o.dn_states_ref_layout().cuda(),
                         o.conv_ref_layout().cuda(), L, int(ids[L]))
        lg = o.step(int(ids[L]))
        tr = torch.stack(o.trace)
        teacher[1:, b] = tr[:-1]
        oracles.append(o); traces.append(tr); ref_logits.append(lg.float()); nxt.append(int(lg.argmax()))
    dbg = torch.zeros(24, B, 1024, dtype=torch.bfloat16, device="cuda")
    logits = torch.zeros(B, D.vocab, dtype=torch.bfloat16, device="cuda")
    toks = bd.step(dbg_hidden=dbg, dbg_teacher=teacher.cuda(), logits_out=logits)
    bd.check_status()
    got = dbg.cpu()
    for b, L in enumerate(lens):
        tr = traces[b]
        exact = int((got[:, b] == tr).all(dim=1).sum())
        frac = float((got[:, b] != tr).float().mean())
        max_abs = float((got[:, b].float() - tr.float()).abs().max())
        ld = (logits[b].float().cpu() - ref_logits[b]).abs()
        print(f"seq {b} (context {L}): {exact}/24 layers bit-identical, {frac:.3%} elements differ, max abs {max_abs}, max |dlogit| {float(ld.max()):.4f}")
        # projections run on tensor cores here: their f32 accumulation flips ~6e-4 of the bf16 roundings against the CPU
        # (the FMA GEMV of the bs=1 kernel: ~1e-4), so fewer layers are bit-identical; every element stays within 2^-5
        assert exact >= 2 and frac < FRAC_TOL and max_abs <= LAYER_ABS_TOL
        assert float(ld.max()) <= LOGIT_TOL
        top = torch.topk(ref_logits[b], 2).values
        if float(top[0] - top[1]) > 2 * float(ld.max()):
            assert int(toks[b]) == nxt[b]
        o = oracles[b]
        st, sr = bd.dn_states[b].cpu(), o.dn_states_ref_layout()
        assert float((st - sr).norm() / sr.norm()) <= STATE_REL_TOL
        cv, cr = bd.conv_bufs[b].cpu(), o.conv_ref_layout()
        assert float((cv != cr).float().mean()) < 0.01
        # the appended K/V row of the first attention layer, read back through the page table
        page = int(bd.block_table[b, L // 64])
        k_new = bd.k_pages[0, page, :, L % 64].float().cpu()
        assert float((k_new - torch.stack(o.k_cache)[0, :, L].float()).abs().max()) <= 0.0625
    assert bd.positions.tolist() == [L + 1 for L in lens]


def test_batched_free_running_and_prefill(full_weights_cpu):
    """prefill() installs a sequence with the library's own prefill; a few steps run; equal inputs give equal outputs."""
    from qwen35_b200.config import QWEN35_0P8B as D
    from qwen35_b200.model import BatchedDecoder
    from qwen35_b200.weights import make_token_ids, weights_to
    wg = weights_to(full_weights_cpu, "cuda")
    bd = BatchedDecoder(wg, batch=4, max_ctx=192)
    ids = make_token_ids(40, 5, D.vocab).cuda()
    for b in range(4):
        bd.prefill(b, ids if b != 2 else ids[:33])
    outs = torch.stack([bd.step().clone() for _ in range(6)])      # [steps, batch]
    bd.check_status()
    assert torch.equal(outs[:, 0], outs[:, 1]) and torch.equal(outs[:, 0], outs[:, 3])      # identical sequences stay identical
    assert bool(((outs >= 0) & (outs < D.vocab)).all())
    assert bd.positions.tolist() == [46, 46, 39, 46]


def test_batched_graph_replay_equals_eager(full_weights_cpu):
    """step(graph=True) replays a CUDA graph of the same launches: tokens, positions and states equal the eager run."""
    from qwen35_b200.config import QWEN35_0P8B as D
    from qwen35_b200.model import BatchedDecoder
    from qwen35_b200.weights import make_token_ids, weights_to
    wg = weights_to(full_weights_cpu, "cuda")
    runs = []
    for use_graph in (False, True):
        bd = BatchedDecoder(wg, batch=3, max_ctx=192)
        for b in range(3):
            bd.prefill(b, make_token_ids(20 + 30 * b, 9 + b, D.vocab).cuda())
        outs = torch.stack([bd.step(graph=use_graph).clone() for _ in range(5)])
        bd.check_status()
        runs.append((outs.cpu(), bd.positions.cpu(), bd.dn_states.cpu()))
    assert torch.equal(runs[0][0], runs[1][0]) and torch.equal(runs[0][1], runs[1][1]) and torch.equal(runs[0][2], runs[1][2])


def test_batched_two_concurrent_groups_equal_one_batch(full_weights_cpu):
    """groups=2 runs the two halves of the batch as concurrent sub-batches (two streams, caller-owned scratch per call):
    every sequence's tokens, position and state equal the single-batch run."""
    from qwen35_b200.config import QWEN35_0P8B as D
    from qwen35_b200.model import BatchedDecoder
    from qwen35_b200.weights import make_token_ids, weights_to
    wg = weights_to(full_weights_cpu, "cuda")
    runs = []
    for groups in (1, 2):
        bd = BatchedDecoder(wg, batch=4, max_ctx=192, groups=groups)
        for b in range(4):
            bd.prefill(b, make_token_ids(18 + 25 * b, 3 + b, D.vocab).cuda())
        outs = torch.stack([bd.step(graph=True).clone() for _ in range(5)])
        bd.check_status()
        runs.append((outs.cpu(), bd.positions.cpu(), bd.dn_states.cpu(), bd.conv_bufs.cpu()))
    for a, b in zip(runs[0], runs[1]):
        assert torch.equal(a, b)


def test_batched_64_sequences_with_long_contexts(full_weights_cpu):
    """The benchmarked batch: 64 sequences in one step, two of them at contexts beyond 2048 tokens (17 attention chunks of
    128 positions, 33 KV pages), compared with the bs=1 oracle like the short ones; the other sequences hold short
    contexts and are checked for running in range."""
    from oracle.qwen35_oracle import Oracle
    from qwen35_b200.config import QWEN35_0P8B as D
    from qwen35_b200.model import BatchedDecoder
    from qwen35_b200.weights import make_token_ids, weights_to
    wg = weights_to(full_weights_cpu, "cuda")
    B = 64
    lens = {0: 2049, 63: 2100, 17: 5, 40: 129}
    bd = BatchedDecoder(wg, batch=B, max_ctx=2304)
    teacher = torch.zeros(24, B, 1024, dtype=torch.bfloat16)
    refs = {}
    for b in range(B):
        L = lens.get(b, 1 + b % 7)
        ids = make_token_ids(L + 1, 500 + b, D.vocab)
        o = Oracle(full_weights_cpu, D, 2304)
        o.prefill(ids[:L])
        bd.load_sequence(b, torch.stack(o.k_cache).cuda(), torch.stack(o.v_cache).cuda(), o.dn_states_ref_layout().cuda(),
                         o.conv_ref_layout().cuda(), L, int(ids[L]))
        if b in lens:
            lg = o.step(int(ids[L]))
            tr = torch.stack(o.trace)
            teacher[1:, b] = tr[:-1]
            refs[b] = (o, tr, lg.float(), L)
    dbg = torch.zeros(24, B, 1024, dtype=torch.bfloat16, device="cuda")
    logits = torch.zeros(B, D.vocab, dtype=torch.bfloat16, device="cuda")
    toks = bd.step(dbg_hidden=dbg, dbg_teacher=teacher.cuda(), logits_out=logits)
    bd.check_status()
    got = dbg.cpu()
    for b, (o, tr, ref_lg, L) in refs.items():
        frac = float((got[:, b] != tr).float().mean())
        max_abs = float((got[:, b].float() - tr.float()).abs().max())
        dl = float((logits[b].float().cpu() - ref_lg).abs().max())
        print(f"B=64, seq {b} (context {L}): {frac:.3%} of elements differ, max abs {max_abs}, max |dlogit| {dl:.4f}")
        assert frac < FRAC_TOL and max_abs <= LAYER_ABS_TOL and dl <= LOGIT_TOL
        st, sr = bd.dn_states[b].cpu(), o.dn_states_ref_layout()
        assert float((st - sr).norm() / sr.norm()) <= STATE_REL_TOL
        page = int(bd.block_table[b, L // 64])
        k_new = bd.k_pages[:, page, :, L % 64].float().cpu()                   # the appended K row of all six attention layers
        assert float((k_new - torch.stack(o.k_cache)[:, :, L].float()).abs().max()) <= 0.0625
    assert bool(((toks >= 0) & (toks < D.vocab)).all())
    assert int(bd.positions[0]) == 2050 and int(bd.positions[63]) == 2101


def test_batched_position_beyond_the_cache_is_refused(full_weights_cpu):
    """Positions advance on the device.  The host refuses a step once its own bound reaches max_ctx; a position written
    behind its back is caught by the kernels, which skip that sequence (no K/V write, no advance), leave the others
    alone and set the sticky status word."""
    from qwen35_b200._capi import Qwen35Error
    from qwen35_b200.config import QWEN35_0P8B as D
    from qwen35_b200.model import BatchedDecoder
    from qwen35_b200.weights import make_token_ids, weights_to
    wg = weights_to(full_weights_cpu, "cuda")
    bd = BatchedDecoder(wg, batch=2, max_ctx=64)
    for b in range(2):
        bd.prefill(b, make_token_ids(60, 40 + b, D.vocab).cuda())
    for _ in range(4):
        bd.step()
    bd.check_status()
    assert bd.positions.tolist() == [64, 64]
    with pytest.raises(ValueError):
        bd.step()                                   # the host's bound: position 64 does not fit a 64-token cache
    # behind the host's back: sequence 1 claims a position far outside its page-table row
    bd2 = BatchedDecoder(wg, batch=2, max_ctx=64)
    for b in range(2):
        bd2.prefill(b, make_token_ids(20, 40 + b, D.vocab).cuda())
    ref = BatchedDecoder(wg, batch=2, max_ctx=64)
    for b in range(2):
        ref.prefill(b, make_token_ids(20, 40 + b, D.vocab).cuda())
    k_before = bd2.k_pages.clone()
    bd2.positions[1] = 5000
    t = bd2.step().clone()
    t_ref = ref.step().clone()
    with pytest.raises(Qwen35Error):
        bd2.check_status()
    assert int(bd2.positions[1]) == 5000 and int(bd2.positions[0]) == 21          # skipped sequence did not advance
    assert int(t[0]) == int(t_ref[0])                                              # its neighbour is unaffected
    assert torch.equal(bd2.k_pages[:, 1], k_before[:, 1])                         # nothing written into sequence 1's page
    import ctypes as C
    bd2._lib.qwen35_b200_clear_status(C.c_void_p(torch.cuda.current_stream().cuda_stream))
    bd2.check_status()
