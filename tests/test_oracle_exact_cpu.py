"""The exactly-rounded evaluation of the oracle (every projection summed in f64 and rounded once): the yardstick against
which both the HuggingFace-order oracle and the CUDA path are measured in tests/test_decode_gpu.py.  CPU only."""
import copy

import numpy as np
import torch

import oracle.qwen35_oracle as Q


def test_single_rounding_from_f64():
    # 1 + 2^-8 is the midpoint between bf16(1) and the next bf16 value: ties go to even (1.0); a hair above goes up.
    x = torch.tensor([1.0 + 2.0 ** -8, 1.0 + 2.0 ** -8 + 2.0 ** -40, 1.0 + 3 * 2.0 ** -8, -(1.0 + 2.0 ** -8 + 2.0 ** -50)], dtype=torch.float64)
    got = Q.f64_to_bf16_once(x).float().tolist()
    assert got == [1.0, 1.0 + 2.0 ** -7, 1.0 + 2.0 ** -6, -(1.0 + 2.0 ** -7)]
    # the classic double-rounding case: a value just above a bf16 midpoint that f32 rounding would pull onto the midpoint
    y = torch.tensor([1.0 + 2.0 ** -8 + 2.0 ** -30], dtype=torch.float64)
    assert float(y.to(torch.float32).to(torch.bfloat16)) == 1.0            # two roundings: wrong
    assert float(Q.f64_to_bf16_once(y)) == 1.0 + 2.0 ** -7                 # one rounding: right


def test_hf_order_oracle_sits_close_to_the_exact_evaluation():
    """On the tiny configuration: a teacher-forced decode step of the oracle in torch's f32 summation order differs from
    the exactly-rounded evaluation in a small share of the layer outputs, each by a last place or two."""
    from qwen35_b200.config import TINY
    from qwen35_b200.weights import make_random_weights, make_token_ids
    w = make_random_weights(5, TINY)
    ids = make_token_ids(9, 3, TINY.vocab)
    o = Q.Oracle(w, TINY, 64)
    o.prefill(ids[:8])
    oe = copy.deepcopy(o)
    o.step(int(ids[8]))
    trace = torch.stack(o.trace)
    teacher = [None] + [trace[i][None] for i in range(len(trace) - 1)]
    Q.EXACT_LINEAR = True
    try:
        oe.step(int(ids[8]), teacher=teacher)
    finally:
        Q.EXACT_LINEAR = False
    exact = torch.stack(oe.trace)
    frac = float((exact != trace).float().mean())
    assert frac < 0.10
    assert float((exact.float() - trace.float()).abs().max()) <= 2.0 ** -5
    # and the exact mode is really another evaluation, not the same code path
    a = torch.randn(4, 3584).bfloat16(); b = (torch.randn(64, 3584) * 0.1).bfloat16()
    Q.EXACT_LINEAR = True
    try:
        e = Q.linear(a, b)
    finally:
        Q.EXACT_LINEAR = False
    ref = torch.from_numpy(np.asarray(a.double().numpy() @ b.double().numpy().T)).float()
    assert float((e.float() - ref).abs().max()) <= float(ref.abs().max()) * 2.0 ** -8
