"""GPU parity of the prompt pass with NVFP4 operands: the fused projection and gate/up GEMMs of every layer and the LM head
run block-scaled on the tensor cores (tcgen05 kind::mxf4nvf4), activations quantised per 16-element block on the way.

The oracle takes the same projections on the same operands: the weight bytes the GPU packer wrote, dequantised on the CPU,
and activations quantised by the CPU restatement of the activation quantiser; sums in f64, one rounding to bf16.  All other
operations are the bf16 oracle's.  Teacher forced like the bf16 sweep test, so each layer is compared on its own.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LAYER_ABS_TOL = 2.0 ** -5
STATE_REL_TOL = 1e-3
LOGIT_TOL = 2e-2


def _dequant(packed, scales, rows):
    from oracle.nvfp4_ref import dequantize_nvfp4_lm
    return torch.from_numpy(dequantize_nvfp4_lm(packed.cpu().numpy(), scales.cpu().numpy())[:rows].copy())


def _oracle_table(w_cpu, w_gpu, D, with_lm=True):
    """{id(cpu weight): dequantised copy of what the GPU packed for it}, for the matrices the NVFP4 prompt pass quantises."""
    table = {}
    for ld, f in zip(w_cpu["layer_data"], w_gpu["prefill_fused_layer_data"]):
        p = ld["ptrs"]
        proj = _dequant(f["proj_weight_packed"], f["proj_weight_scales"], f["proj_weight"].shape[0])
        gu = _dequant(f["gate_up_weight_packed"], f["gate_up_weight_scales"], f["gate_up_weight"].shape[0])
        parts = [p[1], p[2], p[3], p[4]] if ld["type"] == 0 else [p[1], p[2], p[3]]
        gate, up = (p[11], p[12]) if ld["type"] == 0 else (p[8], p[9])
        r = 0
        for t in parts:
            table[id(t)] = proj[r:r + t.shape[0]]
            r += t.shape[0]
        assert r == f["proj_weight"].shape[0]
        table[id(gate)], table[id(up)] = gu[:gate.shape[0]], gu[gate.shape[0]:]
    if with_lm:
        lm = w_gpu["prefill_lm_nvfp4"]
        table[id(w_cpu["lm_head_weight"])] = _dequant(lm["packed"], lm["scales"], D.vocab)
    return table


@pytest.fixture(scope="module")
def nv(full_weights_cpu):
    import oracle.qwen35_oracle as om
    from qwen35_b200.config import QWEN35_0P8B as D
    from qwen35_b200.model import Decoder
    from qwen35_b200.weights import weights_to
    w_gpu = weights_to(full_weights_cpu, "cuda")
    dec = Decoder(weights=w_gpu, max_seq_len=512, prefill_nvfp4=True)
    table = _oracle_table(full_weights_cpu, w_gpu, D)
    yield dict(D=D, dec=dec, w=full_weights_cpu, w_gpu=w_gpu, table=table, om=om)
    om.NVFP4_LINEAR = None


def test_packed_prompt_matrices_follow_the_reference_packer(nv):
    """The fused matrices' packed bytes and scale atoms equal the CPU restatement of the reference's tensor-core packer up to
    the neighbouring-code cases of the approximate reciprocal (the packer is compiled like the reference's, with fast math)."""
    from oracle.nvfp4_ref import quantize_nvfp4_lm
    f = nv["w_gpu"]["prefill_fused_layer_data"][0]
    w = f["gate_up_weight"].float().cpu().numpy()
    packed, scales = quantize_nvfp4_lm(w)
    got_p, got_s = f["gate_up_weight_packed"].cpu().numpy(), f["gate_up_weight_scales"].cpu().numpy()
    assert (got_s != scales).mean() < 1e-3
    assert (got_p != packed).mean() < 1e-3
    # the DeltaNet projection is padded from 8224 to 8320 rows with zeros: codes 0, scale = encoding of 2^-28 saturated up
    pp = f["proj_weight_packed"]
    assert pp.shape[0] == 8320 and int(pp[8224:].max()) == 0


def test_prefill_nvfp4_teacher_forced(nv):
    """All 24 layers at S = 512, every layer on the oracle's input for it: last-position outputs, DeltaNet states, the
    logits of the FP4 head from the GPU's own last hidden row, and the token."""
    from qwen35_b200.weights import make_token_ids
    D, dec, om = nv["D"], nv["dec"], nv["om"]
    S = 512
    ids = make_token_ids(S, 31, D.vocab)
    om.NVFP4_LINEAR = nv["table"]
    try:
        o = om.Oracle(nv["w"], D, S)
        o.keep_all = True
        ref_logits = o.prefill(ids).float()
        teacher = torch.zeros(24, S, 1024, dtype=torch.bfloat16)
        for l in range(1, 24):
            teacher[l] = o.trace_all[l - 1]
        dbg = torch.zeros(24, 1024, dtype=torch.bfloat16, device="cuda")
        logits = torch.zeros(D.vocab, device="cuda")
        tok = dec.prefill_tokens(ids.cuda(), logits_out=logits, dbg_teacher=teacher.cuda(), dbg_hidden=dbg)
        dec.check_status()
        trace = torch.stack(o.trace)
        got = dbg.cpu()
        frac = float((got != trace).float().mean())
        max_abs = float((got.float() - trace.float()).abs().max())
        # the logits the oracle computes from the GPU's own last hidden row: the FP4 head alone
        head_ref = o.logits_from_hidden(got[23][None])[0].float()
        dl_head = float((logits.cpu() - head_ref).abs().max())
        dl = float((logits.cpu() - ref_logits).abs().max())
        st, sr = dec._dn_states.cpu(), o.dn_states_ref_layout()
        rel = max(float((st[i] - sr[i]).norm() / sr[i].norm()) for i in range(18))
        print(f"NVFP4 prefill S={S} teacher forced: {frac:.3%} of last-position elements differ, max abs {max_abs}, "
              f"FP4 head max |dlogit| {dl_head:.4f} (whole pass {dl:.4f}), worst DeltaNet state rel error {rel:.2e}")
        assert max_abs <= LAYER_ABS_TOL and frac < 0.18
        assert dl_head <= LOGIT_TOL and dl <= LOGIT_TOL
        assert rel <= STATE_REL_TOL
        top = torch.topk(head_ref, 2).values
        if float(top[0] - top[1]) > 2 * dl_head:
            assert tok == int(head_ref.argmax())
    finally:
        om.NVFP4_LINEAR = None


def test_fp4_head_token_is_lowest_index_argmax(nv):
    """The token equals the arg-max of the logits the pass wrote, the lowest index among equal maxima (the reference's
    lm_head_kernel_nvfp4 reduction order, kernel_gb10_nvfp4.cu:1451-1523)."""
    from qwen35_b200.weights import make_token_ids
    D, dec = nv["D"], nv["dec"]
    for seed in (3, 4, 5):
        ids = make_token_ids(70 + seed, seed, D.vocab).cuda()
        logits = torch.zeros(D.vocab, device="cuda")
        tok = dec.prefill_tokens(ids, logits_out=logits)
        dec.check_status()
        m = logits.max()
        assert tok == int((logits == m).nonzero()[0])


def test_bf16_decoder_ignores_fp4_copies_in_the_weights(nv):
    """A second decoder on the same weights without the option runs the bf16 GEMMs although the weights now carry FP4 copies."""
    from qwen35_b200.model import Decoder
    from qwen35_b200.weights import make_token_ids
    D = nv["D"]
    ids = make_token_ids(100, 9, D.vocab).cuda()
    d16 = Decoder(weights=nv["w_gpu"], max_seq_len=128)
    h16 = torch.zeros(24, 1024, dtype=torch.bfloat16, device="cuda"); h4 = torch.zeros_like(h16)
    l16, l4 = torch.zeros(D.vocab, device="cuda"), torch.zeros(D.vocab, device="cuda")
    d16.prefill_tokens(ids, logits_out=l16, dbg_num_layers=1, dbg_hidden=h16)
    nv["dec"].prefill_tokens(ids, logits_out=l4, dbg_num_layers=1, dbg_hidden=h4)
    # against a fresh bf16 decoder on weights that never saw the FP4 option
    from qwen35_b200.weights import weights_to
    d_ref = Decoder(weights=weights_to(nv["w"], "cuda"), max_seq_len=128)
    hr = torch.zeros_like(h16); lr = torch.zeros(D.vocab, device="cuda")
    d_ref.prefill_tokens(ids, logits_out=lr, dbg_num_layers=1, dbg_hidden=hr)
    assert torch.equal(h16[0], hr[0])
    assert not torch.equal(h4[0], hr[0])           # FP4 operands change the numbers
    assert float((h4[0].float() - hr[0].float()).abs().max()) < 0.5
