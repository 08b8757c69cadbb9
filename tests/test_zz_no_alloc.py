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


_FRESH_PROCESS = r"""
import ctypes as C, sys
sys.path.insert(0, {root!r}); sys.path.insert(0, {pkg!r})
import torch
from qwen35_b200 import _capi
from qwen35_b200.config import QWEN35_0P8B as D
from qwen35_b200.model import Decoder
from qwen35_b200.weights import make_random_weights, make_token_ids, weights_to
lib = _capi.lib()
dec = Decoder(weights=weights_to(make_random_weights(1234, D), "cuda"), max_seq_len=256)
ids = make_token_ids(6, 5, D.vocab).cuda()
out = torch.zeros(6, dtype=torch.int32, device="cuda")
stream = dec._stream()

def call(pos):
    a = dec._args(forced_ids=ids.data_ptr(), n_steps=6, out_tokens=out.data_ptr())
    a.position = pos
    _capi.check(lib.qwen35_b200_decode_steps_static(C.byref(a), stream), "decode_steps_static")
    _capi.check(lib.qwen35_b200_status(stream), "status")          # synchronises; must not create the regular workspace

call(0)                                   # first call on the device: module load + symbol look-up happen here
torch.cuda.synchronize()
assert lib.qwen35_b200_workspace_if_any() is None, "status() created the library workspace"
free0, _ = torch.cuda.mem_get_info()
call(6)
_capi.check(lib.qwen35_b200_clear_status(stream), "clear_status")
torch.cuda.synchronize()
free1, _ = torch.cuda.mem_get_info()
assert lib.qwen35_b200_workspace_if_any() is None, "status()/clear_status() created the library workspace"
assert free1 == free0, f"device memory in use changed across an allocation-free call: {{free0}} -> {{free1}}"
print("NOALLOC_OK", out.tolist())
"""


def test_static_entry_point_and_status_allocate_nothing_in_a_fresh_process():
    """A process that only ever uses the allocation-free entry point, and reads and clears the status the way the header tells it
    to, must never make the library allocate: the regular workspace does not come into being and the device's free
    memory is the same before and after a call.  Runs in a child process, because every other test of this session has
    already made the library create its workspace."""
    import os
    import subprocess
    import sys
    from conftest import ROOT
    code = _FRESH_PROCESS.format(root=ROOT, pkg=os.path.join(ROOT, "lucebox-hub_b200"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "NOALLOC_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]
