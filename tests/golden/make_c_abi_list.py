"""Extract the `extern "C"` launcher declarations of the reference's binding layer
(models/qwen35_0p8b/torch_bindings.cpp) into tests/golden/reference_c_abi.json: per function its name and the
parameter list as (type, name) pairs.  tests/test_capi_cpu.py compares the library and include/qwen35_b200.h with it.

Usage (where the reference checkout is present):  python tests/golden/make_c_abi_list.py [/path/to/reference]
"""
import json
import os
import re
import sys


def parse_extern_c(text):
    text = re.sub(r"//[^\n]*", "", text)
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    out = []
    for m in re.finditer(r'extern\s+"C"\s+(\w[\w\s\*]*?)\b(\w+)\s*\(([^)]*)\)\s*;', text, flags=re.S):
        params = []
        for p in m.group(3).split(","):
            p = " ".join(p.split())
            if not p or p == "void":
                continue
            pm = re.match(r"(.*?)(\w+)$", p)
            params.append([pm.group(1).replace(" *", "*").replace("* ", "*").strip(), pm.group(2)])
        out.append({"name": m.group(2), "returns": " ".join(m.group(1).split()), "params": params})
    return out


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    src = os.path.join(ref, "models", "qwen35_0p8b", "torch_bindings.cpp")
    fns = parse_extern_c(open(src).read())
    here = os.path.dirname(os.path.abspath(__file__))
    with open(os.path.join(here, "reference_c_abi.json"), "w") as f:
        json.dump({"source": "models/qwen35_0p8b/torch_bindings.cpp", "functions": fns}, f, indent=1)
    print(len(fns), "functions:", [x["name"] for x in fns])


if __name__ == "__main__":
    main()
