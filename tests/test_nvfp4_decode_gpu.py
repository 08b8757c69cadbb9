"""GPU parity of the NVFP4 decode megakernel: weights packed by the library's own packers, the oracle run on
the dequantised values (f32 weights, bf16 activations) -- layer level, teacher forced, as for bf16 -- plus the
reference-signature entry points launch_decode_nvfp4 / launch_decode_many_nvfp4."""
import ctypes as C

import numpy as np
import pytest
import torch

from helpers import load_oracle_state
from oracle import nvfp4_ref as R

pytestmark = pytest.mark.gpu

LAYER_ABS_TOL = 2.0 ** -5
STATE_REL_TOL = 1e-3
LOGIT_TOL = 2e-2                 # teacher-forced logits: the task's bound


@pytest.fixture(scope="module")
def ctx(full_weights_cpu):
    from qwen35_b200.config import QWEN35_0P8B as D
    from qwen35_b200.model import Decoder
    from qwen35_b200.weights import make_token_ids, weights_to
    wg = weights_to(full_weights_cpu, "cuda")
    dec = Decoder(weights=wg, backend="nvfp4", max_seq_len=512)
    # oracle weights: the packed tensors, dequantised on the CPU by the numpy oracle
    nv = wg["nvfp4"]
    wq = {"embed_weight": full_weights_cpu["embed_weight"], "final_norm_weight": full_weights_cpu["final_norm_weight"], "layer_data": []}
    deq = lambda q: torch.from_numpy(R.dequantize_nvfp4(q["packed"].cpu().numpy(), q["scales"].cpu().numpy(), 32))   # noqa: E731
    for ld, nl in zip(full_weights_cpu["layer_data"], nv["layer_data"]):
        p = list(ld["ptrs"])
        qs = nl["quantized"]
        idx = [1, 2, 3, 6, 8, 9, 10] if ld["type"] == 1 else [1, 2, 9, 11, 12, 13]
        for i, q in zip(idx, qs):
            p[i] = deq(q)
        wq["layer_data"].append({"type": ld["type"], "ptrs": p})
    wq["lm_head_weight"] = torch.from_numpy(R.dequantize_nvfp4_lm(nv["lm_head_weight_packed"].cpu().numpy(), nv["lm_head_scales"].cpu().numpy()))
    return dict(D=D, dec=dec, wq=wq, ids=make_token_ids(48, 7, D.vocab))


@pytest.mark.parametrize("n_prompt", [1, 20])
def test_layer_parity_teacher_forced(ctx, n_prompt):
    from oracle.qwen35_oracle import Oracle
    D, dec, ids = ctx["D"], ctx["dec"], ctx["ids"]
    o = Oracle(ctx["wq"], D, 512)
    o.prefill(ids[:n_prompt])
    load_oracle_state(dec, o)
    ref_logits = o.step(int(ids[n_prompt]))
    trace = torch.stack(o.trace)
    teacher = torch.zeros(24, 1024, dtype=torch.bfloat16)
    teacher[1:] = trace[:-1]
    dbg = torch.zeros(24, 1024, dtype=torch.bfloat16, device="cuda")
    logits = torch.zeros(D.vocab, device="cuda")
    tok = dec.forced_steps(ids[n_prompt:n_prompt + 1].cuda(), logits_out=logits, dbg_hidden=dbg, dbg_teacher=teacher.cuda())
    dec.check_status()
    got = dbg.cpu()
    exact_layers = int((got == trace).all(dim=1).sum())
    frac = float((got != trace).float().mean())
    max_abs = float((got.float() - trace.float()).abs().max())
    ld = (logits.cpu() - ref_logits.float()).abs()
    print(f"nvfp4 n_prompt={n_prompt}: {exact_layers}/24 layers bit-identical, {frac:.4%} elements differ, max abs {max_abs}, max |dlogit| {float(ld.max()):.4f}")
    assert exact_layers >= 14 and frac < 0.06 and max_abs <= LAYER_ABS_TOL
    assert float(ld.max()) <= LOGIT_TOL
    top = torch.topk(ref_logits.float(), 2).values
    if float(top[0] - top[1]) > 2 * float(ld.max()):
        assert int(tok[0]) == int(ref_logits.argmax())
    st, sr = dec._dn_states.cpu(), o.dn_states_ref_layout()
    assert float((st - sr).norm() / sr.norm()) <= STATE_REL_TOL


def test_reference_signature_entry_points(ctx):
    """launch_decode_nvfp4 reads its token from device memory; launch_decode_many_nvfp4 chains steps on the device.
    Both must reproduce what the extended entry point generates."""
    from qwen35_b200 import _capi
    dec = ctx["dec"]
    lib = _capi.lib()
    ids = ctx["ids"][:6].cuda()
    dec.reset()
    first = int(dec.forced_steps(ids)[-1])
    snap = [t.clone() for t in (dec._fa_k_cache, dec._fa_v_cache, dec._dn_states, dec._conv_bufs)]

    def restore():
        for d, s_ in zip((dec._fa_k_cache, dec._fa_v_cache, dec._dn_states, dec._conv_bufs), snap):
            d.copy_(s_)
        dec._position = 6

    restore()
    ref = dec.step_many(first, 5).tolist()
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    common = lambda: [dec._embed_weight.data_ptr(), dec._layer_weights_packed_nvfp4.data_ptr(), dec._final_norm_weight.data_ptr(),   # noqa: E731
                      dec._lm_head_weight_packed.data_ptr(), dec._lm_head_scales.data_ptr(), None, None, None, None,
                      dec._fa_k_cache.data_ptr(), dec._fa_v_cache.data_ptr(), dec._dn_states.data_ptr(), dec._conv_bufs.data_ptr(),
                      dec._hidden.data_ptr()] + [None] * 10 + [None] * 5
    # one step at a time, token fed back through the device buffer
    restore()
    tokbuf = torch.tensor([first], dtype=torch.int32, device="cuda")
    got = []
    for i in range(5):
        _capi.check(lib.launch_decode_nvfp4(tokbuf.data_ptr(), tokbuf.data_ptr(), *common(), 6 + i, dec.max_seq_len, 32, st), "launch_decode_nvfp4")
        got.append(int(tokbuf.item()))
    assert got == ref
    # five steps in one launch
    restore()
    tokbuf = torch.tensor([first], dtype=torch.int32, device="cuda")
    outs = torch.zeros(5, dtype=torch.int32, device="cuda")
    _capi.check(lib.launch_decode_many_nvfp4(tokbuf.data_ptr(), outs.data_ptr(), 5, *common(), 6, dec.max_seq_len, 32, st), "launch_decode_many_nvfp4")
    dec.check_status()
    assert outs.tolist() == ref and int(tokbuf.item()) == ref[-1]
    with pytest.raises(_capi.Qwen35Error):
        _capi.check(lib.launch_decode_nvfp4(tokbuf.data_ptr(), tokbuf.data_ptr(), *common(), 11, dec.max_seq_len, 16, st), "group 16")


def test_launch_prefill_megakernel_nvfp4(ctx):
    """The reference's argument list (torch_bindings.cpp:104-119): the prompt in one dispatch, token-serial, LM head after
    the last token.  Must leave the state and return the token of the extended entry point run over the same prompt."""
    from qwen35_b200 import _capi
    dec = ctx["dec"]
    lib = _capi.lib()
    ids = ctx["ids"][:9].cuda()
    dec.reset()
    ref_first = int(dec.forced_steps(ids)[-1])
    ref_state, ref_k = dec._dn_states.clone(), dec._fa_k_cache[:, :, :9].clone()
    dec.reset()
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = [ids.data_ptr(), 9, out.data_ptr(), dec._embed_weight.data_ptr(), dec._layer_weights_packed_nvfp4.data_ptr(),
            dec._final_norm_weight.data_ptr(), dec._lm_head_weight_packed.data_ptr(), dec._lm_head_scales.data_ptr(), None, None, None, None,
            dec._fa_k_cache.data_ptr(), dec._fa_v_cache.data_ptr(), dec._dn_states.data_ptr(), dec._conv_bufs.data_ptr(),
            dec._hidden.data_ptr()] + [None] * 10 + [None] * 5 + [dec.max_seq_len, 32, st]
    _capi.check(lib.launch_prefill_megakernel_nvfp4(*args), "launch_prefill_megakernel_nvfp4")
    dec.check_status()
    assert int(out.item()) == ref_first
    assert torch.equal(dec._dn_states, ref_state) and torch.equal(dec._fa_k_cache[:, :, :9], ref_k)
    args[-2] = 16
    with pytest.raises(_capi.Qwen35Error):
        _capi.check(lib.launch_prefill_megakernel_nvfp4(*args), "group 16")
