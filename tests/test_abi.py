"""CPU-side checks of the C ABI: the in-tree library loads, exports every
entry point declared in include/*.h, and fails cleanly without a GPU."""
import ctypes
import glob
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    from mimo_prismwing_b200._lib import header_symbols
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        names.update(header_symbols(h))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    from mimo_prismwing_b200._lib import LIB_PATH
    assert os.path.exists(LIB_PATH), "build with python -m mimo_prismwing_b200.build"
    out = subprocess.run(["nm", "-D", "--defined-only", LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing
    assert len(declared_symbols()) >= 17


def test_library_loads_and_reports_abi_version():
    import mimo_prismwing_b200 as m
    L = m.load()
    assert L.pw_abi_version() == 2


def test_router_descriptor_layout_matches_header():
    # pw_router {const void *weight; const float *bias; uint32_t experts, hidden,
    # top_k, weight_dtype;} and the dtype codes of include/pw_cuda.h
    import re
    from mimo_prismwing_b200 import _lib
    from mimo_prismwing_b200.runtime import ROUTER_BF16, ROUTER_F32, Router
    assert [f[0] for f in Router._fields_] == ["weight", "bias", "experts", "hidden", "top_k", "weight_dtype"]
    assert ctypes.sizeof(Router) == 32
    text = open(_lib.HEADER).read()
    assert int(re.search(r"#define PW_ROUTER_F32 (\d+)u", text).group(1)) == ROUTER_F32
    assert int(re.search(r"#define PW_ROUTER_BF16 (\d+)u", text).group(1)) == ROUTER_BF16


def test_null_and_no_device_paths_fail_cleanly():
    import torch
    import mimo_prismwing_b200 as m
    L = m.load()
    assert L.pw_runtime_create(0, 0, None) == -1
    assert L.pw_synchronize(None) == -1
    assert L.pw_last_error(None) == b"null runtime"
    if not torch.cuda.is_available():
        rt = ctypes.c_void_p()
        st = L.pw_runtime_create(0, 0, ctypes.byref(rt))
        assert st in (-5, -9) and not rt.value


def test_python_mirror_keeps_reference_method_names():
    from mimo_prismwing_b200.runtime import WideMoeRuntime
    for name in ["compile", "compile_with_fused_gate_up", "execute_fp8_linear", "execute", "execute_fused_gate_up"]:
        assert hasattr(WideMoeRuntime, name)


def test_smoke_inputs_build_on_the_host():
    # smoke() builds its bank and router on the host and copies them over with
    # synth.to_device: the same calls with the host as the target
    from mimo_prismwing_b200 import synth
    w, bias = synth.to_device(synth.router(16, 1024, 7, "cpu"), "cpu")
    assert tuple(w.shape) == (16, 1024) and tuple(bias.shape) == (16,)
    gate, up, down = synth.to_device(synth.expert(1024, 512, 100, "cpu"), "cpu")
    assert tuple(gate.weight.shape) == (512, 1024) and tuple(down.weight.shape) == (1024, 512)
