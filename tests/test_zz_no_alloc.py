"""The allocation-free expert entry point (pw_expert_forward_static).

Some callers cannot allocate device memory when they call in (a reserved
memory budget, a host application that owns the allocator, a serving loop
that must not hit cudaMalloc's device synchronisation).  For them the library
offers one entry point whose scratch is a fixed device array inside the
library.  This test calls it through the C ABI and checks it against the
regular pw_expert_forward, on two calls in a row (the second reuses the
array the first left behind).  The file name makes pytest collect it last.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bind():
    import mimo_prismwing_b200 as m
    L = m.load()
    f = L.pw_expert_forward_static
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


def test_static_scratch_expert_matches_allocating_entry_point():
    import torch
    from mimo_prismwing_b200 import synth
    from mimo_prismwing_b200.runtime import ExpertWeights, WideMoeRuntime
    from gpu_helpers import assert_close_bf16

    static_forward = _bind()
    rt = WideMoeRuntime.compile_with_fused_gate_up(0)
    g, u, d = synth.expert(4096, 2048, 77, "cuda")
    weights = ExpertWeights(g.c(), u.c(), d.c())
    for call, width in enumerate([8, 3]):
        x = synth.activations(width, 4096, 700 + call, "cuda")
        ref = rt.expert_forward(x, g, u, d).output.cpu().numpy()
        y = torch.full((width, 4096), float("nan"), device="cuda")
        torch.cuda.synchronize()
        st = static_forward(ctypes.byref(weights), ctypes.c_void_p(x.data_ptr()), width,
                            ctypes.c_void_p(y.data_ptr()), None)
        assert st == 0, f"call {call}: status {st}"
        got = y.cpu().numpy()
        assert np.all(np.isfinite(got))
        assert_close_bf16(got, ref, what=f"static-scratch call {call}")
        # the same kernels in the same order: identical bits
        assert np.array_equal(got, ref)
    rt.close()


def test_static_scratch_expert_allocates_no_device_memory():
    # the property the entry point exists for: once a first round of calls
    # has looked up the array's address and loaded each width's kernels
    # (CUDA loads kernels lazily, on first launch), further calls at every
    # width leave the device's free memory and torch's pool unchanged
    import torch
    from mimo_prismwing_b200 import synth
    from mimo_prismwing_b200.runtime import ExpertWeights

    static_forward = _bind()
    g, u, d = synth.expert(4096, 2048, 79, "cuda")
    weights = ExpertWeights(g.c(), u.c(), d.c())
    xs = [synth.activations(w, 4096, 800 + w, "cuda") for w in range(1, 9)]
    ys = [torch.empty((w, 4096), device="cuda") for w in range(1, 9)]
    for w in range(1, 9):
        assert static_forward(ctypes.byref(weights), ctypes.c_void_p(xs[w - 1].data_ptr()), w,
                              ctypes.c_void_p(ys[w - 1].data_ptr()), None) == 0
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    reserved0 = torch.cuda.memory_reserved()
    for w in range(1, 9):
        assert static_forward(ctypes.byref(weights), ctypes.c_void_p(xs[w - 1].data_ptr()), w,
                              ctypes.c_void_p(ys[w - 1].data_ptr()), None) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"device free memory changed by {free0 - free1} bytes"
    assert torch.cuda.memory_reserved() == reserved0


def test_static_scratch_expert_rejects_sizes_beyond_its_array():
    import torch
    from mimo_prismwing_b200 import synth
    from mimo_prismwing_b200.runtime import ExpertWeights

    static_forward = _bind()
    g, u, d = synth.expert(256, 256, 78, "cuda")
    weights = ExpertWeights(g.c(), u.c(), d.c())
    x = torch.zeros((9, 256), device="cuda")
    y = torch.zeros((9, 256), device="cuda")
    assert static_forward(ctypes.byref(weights), ctypes.c_void_p(x.data_ptr()), 9,
                          ctypes.c_void_p(y.data_ptr()), None) == -9  # PW_ERR_UNSUPPORTED
