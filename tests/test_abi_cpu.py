"""Host-side checks that need no GPU: the C-ABI libraries load and export
every symbol the headers declare, the spec parser (C++) agrees with the
Python one and with the reference's weight layouts, and the configuration
specs on disk match neuralscript_b200.spec."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import neuralscript_b200 as nsb
from neuralscript_b200.spec import CONFIGS, parse
from specs import SMALL

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions(name):
    text = open(os.path.join(ROOT, "include", name)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b((?:ns|nsb|nsb_op)_[a-z0-9_]+)\s*\(", text)))


def exported(path):
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    return {l.split()[-1] for l in out.splitlines() if " T " in l}


def test_core_library_exports_all_declared_functions():
    syms = exported(nsb.CORE_LIB)
    for h in ("ns_b200.h", "ns_b200_ops.h"):
        missing = [f for f in header_functions(h) if f not in syms]
        assert not missing, (h, missing)


@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_model_library_exports_the_reference_abi(name):
    path = os.path.join(nsb.LIB_DIR, f"libns_{name}.so")
    syms = exported(path)
    missing = [f for f in header_functions("ns_runtime.h") if f not in syms]
    assert not missing, missing
    L = nsb.RuntimeLib(name)
    assert L.ns_weight_count_static() == parse(CONFIGS[name]).weight_count


def test_spec_files_match_python_specs():
    for k, v in CONFIGS.items():
        assert open(os.path.join(ROOT, "neuralscript_b200", "specs", f"{k}.nss")).read() == v


@pytest.mark.parametrize("text", list(CONFIGS.values()) + list(SMALL.values()))
def test_cpp_and_python_spec_layouts_agree(text):
    lay = nsb.spec_layout(text)
    py = [(n, o, c) for n, o, c, _ in parse(text).layout()]
    assert lay == py
    assert nsb.lib().nsb_spec_weight_count(text.encode()) == parse(text).weight_count


REF = os.path.join(ROOT, "oracle", "_ref")


@pytest.mark.skipif(not os.path.isdir(REF), reason="reference build absent")
@pytest.mark.parametrize("name,text", [("c1", CONFIGS["c1"]), ("c2", CONFIGS["c2"]), ("c3", CONFIGS["c3"]),
                                       ("tmlp", SMALL["tmlp"]), ("ttfm", SMALL["ttfm"]), ("tmoe", SMALL["tmoe"])])
def test_layout_matches_reference_runtime(name, text):
    """Names, offsets and counts equal the reference's ns_model_layout."""
    path = os.path.join(REF, f"libref_{name}.so")
    if not os.path.exists(path):
        pytest.skip("reference library not built")
    L = C.CDLL(path)
    L.ns_model_layout.restype = C.POINTER(nsb._Layout)
    L.ns_model_layout.argtypes = [C.c_void_p]
    lay = L.ns_model_layout(None).contents
    ref = [(lay.desc[i].name.decode(), lay.desc[i].offset, lay.desc[i].count) for i in range(lay.num_weights)]
    assert nsb.spec_layout(text) == ref


def test_bad_specs_are_rejected():
    assert nsb.lib().nsb_spec_weight_count(b"network X\ninput 4\ny = nothere(x)\n") == 0
    assert "unknown" in nsb.last_error()
    assert nsb.lib().nsb_spec_weight_count(b"network X\ninput 4\nlayer f dense in=5 out=2\ny = f(x)\n") == 0
    assert "mismatch" in nsb.last_error()


def test_no_device_calls_without_gpu_fail_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    w = np.zeros(parse(SMALL["tmlp"]).weight_count, np.float32)
    with pytest.raises(RuntimeError):
        nsb.Model(SMALL["tmlp"], w)
