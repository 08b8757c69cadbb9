"""CPU-side checks of the drop-in boundary: the C-ABI library loads, exports every symbol
include/qwen35_b200.h declares, and the host-side helpers mirror the reference's layouts.
No compute call is made (there is no GPU where these run)."""
import ctypes
import os
import re
import struct

import pytest
import torch

from conftest import ROOT
from qwen35_b200 import _capi
from qwen35_b200.config import QWEN35_0P8B, TINY
from qwen35_b200.weights import make_random_weights, make_token_ids


def _declared_functions():
    text = open(os.path.join(ROOT, "include", "qwen35_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?(?:int|long long|size_t|char\s*\*|void)\s*\*?\s*(\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    names = _declared_functions()
    assert "launch_decode" in names and "qwen35_b200_decode_steps" in names
    lib = ctypes.CDLL(_capi.LIB_PATH)
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/qwen35_b200.h but not exported"
    assert set(_capi.SIGNATURES) <= set(names)


def test_rope_table_matches_torch():
    buf = (ctypes.c_float * 32)()
    assert _capi.lib().qwen35_b200_rope_inv_freq(buf) == 0
    ref = 1.0 / (1.0e7 ** (torch.arange(0, 64, 2, dtype=torch.int64).to(torch.float) / 64))
    assert torch.equal(torch.tensor(list(buf)), ref)


def test_layer_record_layout():
    """128-byte records {int type; int pad[3]; void* ptrs[14]} (reference model.py:410-427)."""
    from qwen35_b200.model import _pack_layer_weights
    w = make_random_weights(1, TINY)
    blob = _pack_layer_weights(w["layer_data"], device="cpu")
    assert blob.numel() == TINY.num_layers * 128
    raw = bytes(blob.numpy())
    for i, ld in enumerate(w["layer_data"]):
        t, p0, p1, p2 = struct.unpack_from("iiii", raw, i * 128)
        assert (t, p0, p1, p2) == (ld["type"], 0, 0, 0)
        ptrs = struct.unpack_from("14Q", raw, i * 128 + 16)
        n = len(ld["ptrs"])
        assert n == (11 if ld["type"] == 1 else 14)
        assert list(ptrs[:n]) == [x.data_ptr() for x in ld["ptrs"]]
        assert all(v == 0 for v in ptrs[n:])


def test_weights_are_reproducible_and_shaped():
    a = make_random_weights(7, TINY)
    b = make_random_weights(7, TINY)
    assert torch.equal(a["embed_weight"], b["embed_weight"])
    assert a["lm_head_weight"] is a["embed_weight"]           # tied (reference model.py:384)
    d = TINY
    dn = next(l for l in a["layer_data"] if l["type"] == 0)["ptrs"]
    fa = next(l for l in a["layer_data"] if l["type"] == 1)["ptrs"]
    assert dn[1].shape == (d.dn_conv_channels, d.hidden) and dn[5].shape == (d.dn_conv_channels, 1, 4)
    assert fa[1].shape == (2 * d.fa_q_size, d.hidden) and fa[6].shape == (d.hidden, d.fa_q_size)
    assert make_token_ids(5, 3, 100).dtype == torch.int32
    assert QWEN35_0P8B.layer_types == [0, 0, 0, 1] * 6


def test_calls_fail_loudly_without_a_device():
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    st = _capi.lib().qwen35_b200_status(None)
    assert st != 0
    with pytest.raises(_capi.Qwen35Error):
        _capi.check(st, "status")


def _header_params():
    """name -> parameter count of every function include/qwen35_b200.h declares."""
    text = open(os.path.join(ROOT, "include", "qwen35_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    out = {}
    for m in re.finditer(r"^\s*(?:const\s+)?(?:int|long long|size_t|char\s*\*|void)\s*\*?\s*(\w+)\s*\(([^)]*)\)\s*;", text, flags=re.M | re.S):
        params = [p for p in (" ".join(x.split()) for x in m.group(2).split(",")) if p and p != "void"]
        out[m.group(1)] = params
    return out


def test_every_reference_launcher_is_exported_with_its_argument_list():
    """The `extern "C"` functions the reference's binding layer declares (torch_bindings.cpp:47-119, 323-364; list kept
    in tests/golden/reference_c_abi.json by make_c_abi_list.py): each is exported by the library and declared in the
    header with the same number of parameters, pointer parameters in the same places."""
    import json
    ref = json.load(open(os.path.join(ROOT, "tests", "golden", "reference_c_abi.json")))["functions"]
    assert len(ref) == 9
    hdr = _header_params()
    lib = ctypes.CDLL(_capi.LIB_PATH)
    for fn in ref:
        name = fn["name"]
        assert hasattr(lib, name), f"{name}: declared by the reference's torch_bindings.cpp, not exported"
        assert name in hdr, f"{name}: not declared in include/qwen35_b200.h"
        assert len(hdr[name]) == len(fn["params"]), f"{name}: {len(hdr[name])} parameters here, {len(fn['params'])} in the reference"
        for mine, (rtype, rname) in zip(hdr[name], fn["params"]):
            if rtype == "cudaStream_t":
                assert mine.startswith("qwen35_stream_t"), f"{name}: parameter {rname}: '{mine}' is not the stream"
            else:
                assert ("*" in mine) == ("*" in rtype), f"{name}: parameter {rname}: '{mine}' vs '{rtype}'"
        assert len(_capi.SIGNATURES[name][1]) == len(fn["params"]), f"{name}: ctypes signature length"


def test_reference_c_abi_fixture_is_current():
    """Where the reference checkout is present, the committed list equals a fresh parse of its binding layer."""
    src = "/root/reference/models/qwen35_0p8b/torch_bindings.cpp"
    if not os.path.exists(src):
        pytest.skip("reference checkout not present")
    import importlib.util
    import json
    spec = importlib.util.spec_from_file_location("make_c_abi_list", os.path.join(ROOT, "tests", "golden", "make_c_abi_list.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    fresh = mod.parse_extern_c(open(src).read())
    assert fresh == json.load(open(os.path.join(ROOT, "tests", "golden", "reference_c_abi.json")))["functions"]
