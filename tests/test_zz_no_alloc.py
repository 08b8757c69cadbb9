"""The allocation-free decode entry point (qwen35_b200_decode_steps_static) against the regular one.

Some hosts of this library may not allocate device memory after start-up -- a serving runtime that has
given all of HBM to its own pool, or a latency-critical loop that cannot afford the device-wide stall of
cudaMalloc.  For them the decode megakernel can run on a fixed scratch array compiled into the library.
The test calls that entry point through the C ABI twice in a row (the second call finds the first call's
words in the shared array) and requires exactly the tokens, logits and state the allocating entry point
produces from the same start state.  This file sorts last so that a run stopping at the first failure
has already executed every other test.
"""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


def _run(dec, entry, first_token, n_steps, logits):
    from qwen35_b200 import _capi
    out = torch.zeros(n_steps, dtype=torch.int32, device=dec.device)
    a = dec._args(token_imm=int(first_token), n_steps=n_steps, out_tokens=out.data_ptr(), logits_out=logits.data_ptr())
    with torch.cuda.device(dec.device):
        _capi.check(entry(C.byref(a), dec._stream()), "decode")
    dec._position += n_steps
    return out


def test_static_scratch_entry_point_matches_allocating_one(full_weights_cpu):
    from qwen35_b200 import _capi
    from qwen35_b200.config import QWEN35_0P8B as D
    from qwen35_b200.model import Decoder
    from qwen35_b200.weights import make_token_ids, weights_to
    lib = _capi.lib()
    dec = Decoder(weights=weights_to(full_weights_cpu, "cuda"), max_seq_len=256)
    ids = make_token_ids(24, 5, D.vocab).cuda()
    first = dec.prefill_tokens(ids)
    snap = [t.clone() for t in (dec._fa_k_cache, dec._fa_v_cache, dec._dn_states, dec._conv_bufs)]

    def restore():
        for dst, src in zip((dec._fa_k_cache, dec._fa_v_cache, dec._dn_states, dec._conv_bufs), snap):
            dst.copy_(src)
        dec._position = 24

    la, lb = torch.zeros(D.vocab, device="cuda"), torch.zeros(D.vocab, device="cuda")
    restore()
    ref1 = _run(dec, lib.qwen35_b200_decode_steps, first, 6, la)
    ref2 = _run(dec, lib.qwen35_b200_decode_steps, int(ref1[-1]), 5, la)
    ref_state = dec._dn_states.clone()
    ref_logits = la.clone()
    restore()
    got1 = _run(dec, lib.qwen35_b200_decode_steps_static, first, 6, lb)          # first call: resolves the symbol address
    got2 = _run(dec, lib.qwen35_b200_decode_steps_static, int(got1[-1]), 5, lb)  # second call: shared array holds call one's words
    dec.check_status()
    assert got1.tolist() == ref1.tolist()
    assert got2.tolist() == ref2.tolist()
    assert torch.equal(lb, ref_logits)                  # same kernel, same arithmetic: bit-identical
    assert torch.equal(dec._dn_states, ref_state)

    # sizes beyond what the array is built for are refused with a message that names the limit
    a = dec._args(token_imm=1, n_steps=1)
    a.max_seq_len = 32768 + 1
    st = lib.qwen35_b200_decode_steps_static(C.byref(a), dec._stream())
    assert st == 2
    assert b"32768" in lib.qwen35_b200_last_error()
