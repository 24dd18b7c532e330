"""GPU parity: the CUDA path through the C ABI against the CPU oracle.

Bit-exact: e4m3 dequantization, dynamic FP8 activation codes and scales,
router logits (pinned f32 slice order), selected expert sets, route weights, the
staged SwiGLU and the weighted combine.  Within relative 2e-3 (norm-wise and
max|d|/max|ref|) of the f64-accumulated oracle: every projection and layer.
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def rt():
    from mimo_prismwing_b200.runtime import WideMoeRuntime
    r = WideMoeRuntime.compile_with_fused_gate_up(0)
    yield r
    r.close()


@pytest.fixture(scope="module")
def rt_unfused():
    from mimo_prismwing_b200.runtime import WideMoeRuntime
    r = WideMoeRuntime.compile(0)
    yield r
    r.close()


def H(t):
    from gpu_helpers import host
    return host(t)


# ------------------------------------------------------------ quantization
def test_dynamic_fp8_matches_pytorch_fixture_bytes(rt):
    with open(os.path.join(GOLDEN, "pw0053_dynamic_fp8.json")) as f:
        fx = json.load(f)
    x = (np.asarray(fx["input_f32_bits"], dtype=np.int64) & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    codes, scales = rt.quantize(torch.from_numpy(x).cuda())
    rows, cols = x.shape
    assert H(codes).reshape(rows, cols // 128, 128).tolist() == fx["encoded_u8"]
    exp_scales = (np.asarray(fx["scale_f32_bits"], dtype=np.int64) & 0xFFFFFFFF).astype(np.uint32)
    assert H(scales).view(np.uint32).tolist() == exp_scales.tolist()


@pytest.mark.parametrize("rows,cols", [(1, 4096), (8, 4096), (37, 2048), (5, 128)])
def test_dynamic_fp8_bit_exact_vs_oracle(rt, rows, cols):
    rng = np.random.default_rng(rows * 1000 + cols)
    x = rng.normal(0, 1, (rows, cols)).astype(np.float32)
    # edge values: zeros, signed zeros, tiny, huge, exact midpoints between codes
    x[0, :128] = 0.0
    x[0, 1] = -0.0
    if cols >= 256:
        x[0, 128:256] = rng.normal(0, 1e-30, 128)
    if rows > 1:
        x[1, :8] = [448.0, -448.0, 1e30, -1e-30, 3.0, 3.25, 3.125, -3.375]
    codes, scales = rt.quantize(torch.from_numpy(x).cuda())
    oc, os_, _ = O.dynamic_fp8(x)
    assert np.array_equal(H(codes), oc)
    assert np.array_equal(H(scales).view(np.uint32), os_.view(np.uint32))
    # host I/O path gives the same bytes
    codes_h, scales_h = rt.quantize(torch.from_numpy(x))
    assert np.array_equal(codes_h.numpy(), oc)


def test_quantize_rejects_nonfinite_and_bad_shape(rt):
    from mimo_prismwing_b200.runtime import PrismwingError
    x = torch.zeros((1, 128), device="cuda")
    x[0, 3] = float("nan")
    with pytest.raises(PrismwingError) as e:
        rt.quantize(x)
    assert e.value.kind == "nonfinite"
    with pytest.raises(PrismwingError) as e:
        rt.quantize(torch.zeros((1, 100), device="cuda"))
    assert e.value.kind == "shape"


# ------------------------------------------------------- readable GEMV (C0)
def test_production_width_real_fp8_gemv_matches(rt):
    # src/lib.rs:8052 fixture through the GPU readable GEMV (tolerance 2e-7)
    from mimo_prismwing_b200.runtime import WideProjectionBinding
    with open(os.path.join(GOLDEN, "mtp_gate_fp8_gemv.json")) as f:
        fx = json.load(f)
    w = np.zeros((128, fx["columns"]), np.uint8)
    w[:fx["rows"]] = np.array(fx["raw_u8"], np.uint8)
    s = np.array(fx["scale_inv"], np.float32).reshape(1, -1)
    b = WideProjectionBinding(torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda())
    x = torch.tensor(fx["input"], dtype=torch.float32).cuda()
    y = H(rt.fp8_gemv(x, b).output)[0, :fx["rows"]]
    assert np.all(np.abs(y - np.array(fx["expected_f32"], np.float32)) < 2e-7)


def test_mapped_fp8_gemv_selects_row_and_column_scale_blocks(rt):
    # src/lib.rs:7807: 256x256 of e4m3 1.0, grid [[1,2],[3,4]], x = 1 -> 384 / 896
    from mimo_prismwing_b200.runtime import WideProjectionBinding
    w = torch.full((256, 256), 0x38, dtype=torch.uint8, device="cuda")
    s = torch.tensor([[1.0, 2.0], [3.0, 4.0]], device="cuda")
    y = H(rt.fp8_gemv(torch.ones(256, device="cuda"), WideProjectionBinding(w, s)).output)[0]
    assert np.all(y[:128] == 384.0) and np.all(y[128:] == 896.0)


def _all_bytes_block():
    """A 128x256 e4m3 block holding every non-NaN byte: W[r, 0] = r and
    W[r, 1] = 128 + r (0x7f and 0xff, the NaNs, left as 0x00), scale 1."""
    w = np.zeros((128, 256), np.uint8)
    w[:, 0] = np.arange(128)
    w[:, 1] = np.arange(128, 256)
    w[0x7F, 0] = 0
    w[0x7F, 1] = 0
    return w, np.ones((1, 2), np.float32)


def test_dequant_all_bytes_bit_exact_on_gpu(rt):
    # src/lib.rs:8012 every_fp8_encoding_matches_oracle, on the GPU: one-hot
    # inputs make y[t, r] = dec(W[r, c_t]) * 1 * 1 exactly, so the readable
    # GEMV's output is the dequantized byte.  Sums start from +0, so the byte
    # 0x80 (-0.0) reads back as +0.0, as in the reference's own projection.
    from mimo_prismwing_b200.runtime import WideProjectionBinding
    with open(os.path.join(GOLDEN, "f8_e4m3fn_all_bytes.json")) as f:
        expected = np.asarray(json.load(f)["expected_f32_bits"], dtype=np.uint32)
    assert len(expected) == 256
    w, s = _all_bytes_block()
    b = WideProjectionBinding(torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda())
    x = torch.zeros((2, 256), device="cuda")
    x[0, 0] = 1.0
    x[1, 1] = 1.0
    y = H(rt.fp8_gemv(x, b).output).view(np.uint32)  # [2, 128]
    got = np.concatenate([y[0], y[1]])                  # byte b at index b
    for byte in range(256):
        if byte in (0x7F, 0xFF):
            continue
        want = expected[byte] if byte != 0x80 else np.uint32(0)
        assert got[byte] == want, f"byte {byte:#04x}: {got[byte]:#010x} != {want:#010x}"


@pytest.mark.parametrize("width", [2, 8, 32])
def test_dequant_all_bytes_through_fp8_mma(rt, width):
    # The block-scaled path feeds the e4m3 bytes to the tensor cores (the
    # tcgen05 GEMV at widths <= 8 for this plain one-tile matrix, the tcgen05
    # GEMM from 32).  With one-hot tokens
    # each output is a single product dec(W) * dec(code) * S * xs, rounded
    # once: bit-exact against the oracle's equation.
    from mimo_prismwing_b200.runtime import WideProjectionBinding
    w, s = _all_bytes_block()
    b = WideProjectionBinding(torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda())
    x = np.zeros((width, 256), np.float32)
    for t in range(width):
        x[t, t % 2 if t < 2 else (t * 37) % 256] = 1.0 if t % 3 else -2.0
    y = H(rt.execute_fp8_linear(torch.from_numpy(x).cuda(), b, f32_output=True).output)
    codes, scales, _ = O.dynamic_fp8(x)
    ref = O.blockscaled_linear(w, s, codes, scales, mode=O.ACC_F32)
    # (+0 canonicalises signed zeros on both sides: a sum from +0 of -0 terms)
    assert np.array_equal((y + np.float32(0)).view(np.uint32), (ref + np.float32(0)).view(np.uint32))
    dec = O.decode_table()
    assert np.array_equal(y[0] != 0, dec[w[:, 0]] != 0) and np.array_equal(y[1] != 0, dec[w[:, 1]] != 0)


@pytest.mark.parametrize("width", [1, 2, 3, 5, 8])
def test_readable_gemv_config0_vs_oracle(rt, width):
    from gpu_helpers import assert_close
    from mimo_prismwing_b200 import synth
    b = synth.projection(2048, 4096, 11, "cuda")
    x = synth.activations(width, 4096, 12 + width, "cuda")
    y = H(rt.fp8_gemv(x, b).output)
    w, s, xn = H(b.weight), H(b.scale), H(x)
    ref = np.stack([O.readable_gemv(w, s, xn[t], O.ACC_F64) for t in range(width)])
    assert_close(y, ref, what=f"readable width {width}")
    # host I/O gives identical bits
    y2 = rt.fp8_gemv(x.cpu(), b).output.numpy()
    assert np.array_equal(y, y2)


# --------------------------------------------------- block-scaled projection
@pytest.mark.parametrize("rows,cols,width", [(2048, 4096, 1), (2048, 4096, 4), (2048, 4096, 8),
                                             (4096, 2048, 2), (4096, 2048, 7), (256, 512, 3),
                                             (2048, 4096, 13), (128, 128, 1)])
def test_fp8_linear_vs_oracle(rt, rows, cols, width):
    from gpu_helpers import assert_close, assert_close_bf16
    from mimo_prismwing_b200 import synth
    b = synth.projection(rows, cols, rows + cols, "cuda")
    x = synth.activations(width, cols, width, "cuda")
    y = H(rt.execute_fp8_linear(x, b).output)
    codes, scales, _ = O.dynamic_fp8(H(x))
    pre = O.blockscaled_linear(H(b.weight), H(b.scale), codes, scales)
    assert np.array_equal(O.round_bf16(y), y)  # the reference's output is bf16-rounded
    assert_close_bf16(y, O.round_bf16(pre), what=f"linear {rows}x{cols} w{width}")
    # the f32 pre-round projection meets max relative 2e-3 outright
    y32 = H(rt.execute_fp8_linear(x, b, f32_output=True).output)
    assert_close(y32, pre, what=f"linear f32 {rows}x{cols} w{width}")
    assert np.array_equal(O.round_bf16(y32), y)


def test_sglang_blockscaled_probe_widths(rt):
    # src/wide_metal_moe.rs:1330 probe inputs (128x256, widths 2, 9, 26, 32)
    from gpu_helpers import assert_close
    from mimo_prismwing_b200.runtime import WideProjectionBinding
    rows, cols = 128, 256
    w = np.array([(i * 37 + 11) % 0x7F for i in range(rows * cols)], np.uint8).reshape(rows, cols)
    s = np.array([0.003 + i * 0.0017 for i in range(2)], np.float32).reshape(1, 2)
    b = WideProjectionBinding(torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda())
    for active in [2, 9, 26, 32]:
        x = np.array([((i * 29 % 401) - 200.0) / 37.0 for i in range(active * cols)], np.float32).reshape(active, cols)
        codes, scales, _ = O.dynamic_fp8(x)
        gc, gs = rt.quantize(torch.from_numpy(x).cuda())
        assert np.array_equal(H(gc), codes) and np.array_equal(H(gs), scales)
        y = H(rt.execute_fp8_linear(torch.from_numpy(x).cuda(), b, f32_output=True).output)
        ref = O.blockscaled_linear(w, s, codes, scales)
        assert_close(y, ref, what=f"probe width {active}")


@pytest.mark.parametrize("width", [1, 8])
def test_full_qkv_layout_vs_oracle(rt, width):
    from gpu_helpers import assert_close
    from mimo_prismwing_b200 import synth
    b = synth.full_qkv(31, "cuda")
    assert tuple(b.scale.shape) == (108, 32)
    x = synth.activations(width, 4096, 40 + width, "cuda")
    y = H(rt.execute_fp8_linear(x, b, full_qkv_layout=True, f32_output=True).output)
    codes, scales, _ = O.dynamic_fp8(H(x))
    ref = O.blockscaled_linear(H(b.weight), H(b.scale), codes, scales, layout=O.LAYOUT_FULL_QKV)
    assert_close(y, ref, what=f"full qkv w{width}")


def test_swa_qkv_layout_vs_oracle(rt):
    from gpu_helpers import assert_close
    from mimo_prismwing_b200 import synth
    b = synth.swa_qkv(32, "cuda")
    x = synth.activations(3, 4096, 50, "cuda")
    y = H(rt.execute_fp8_linear(x, b, f32_output=True).output)  # [14848, 4096] selects the SWA map
    codes, scales, _ = O.dynamic_fp8(H(x))
    ref = O.blockscaled_linear(H(b.weight), H(b.scale), codes, scales, layout=O.LAYOUT_SWA_QKV)
    assert_close(y, ref, what="swa qkv")


def test_projection_rejects_bad_layouts(rt):
    from mimo_prismwing_b200.runtime import PrismwingError, WideProjectionBinding
    from mimo_prismwing_b200 import synth
    b = synth.projection(256, 256, 1, "cuda")
    bad = WideProjectionBinding(b.weight, b.scale[:, :1].contiguous())
    with pytest.raises(PrismwingError) as e:
        rt.execute_fp8_linear(torch.zeros((1, 256), device="cuda"), bad)
    assert e.value.kind == "shape"
    with pytest.raises(PrismwingError) as e:
        rt.execute_fp8_linear(torch.zeros((1, 256), device="cuda"), b, full_qkv_layout=True)
    assert e.value.kind == "shape"
    x = torch.zeros((1, 256), device="cuda")
    x[0, 0] = float("inf")
    with pytest.raises(PrismwingError) as e:
        rt.execute_fp8_linear(x, b)
    assert e.value.kind == "nonfinite"


# ------------------------------------------------------- one expert (C1)
@pytest.mark.parametrize("width", [1, 2, 4, 8])
def test_expert_forward_config1_vs_oracle(rt, width):
    from gpu_helpers import assert_close_bf16, bank_arrays
    from mimo_prismwing_b200 import synth
    g, u, d = synth.expert(4096, 2048, 7, "cuda")
    x = synth.activations(width, 4096, 70 + width, "cuda")
    y = H(rt.expert_forward(x, g, u, d).output)
    (gw, gs, uw, us, dw, ds), = bank_arrays([(g, u, d)])
    xc, xs, _ = O.dynamic_fp8(H(x))
    gate = O.blockscaled_linear(gw, gs, xc, xs)
    up = O.blockscaled_linear(uw, us, xc, xs)
    act = O.staged_swiglu(gate, up, O.EXP_SLEEF)
    hc, hs, _ = O.dynamic_fp8(act)
    ref = O.round_bf16(O.blockscaled_linear(dw, ds, hc, hs))
    assert_close_bf16(y, ref, what=f"expert w{width}")


def test_fused_gate_up_swiglu_is_exact_against_unfused(rt, rt_unfused):
    # src/wide_metal_moe.rs:1343 fused_gate_up_swiglu_is_exact_at_narrow_and_full_expert_widths
    from mimo_prismwing_b200 import synth
    g, u, d = synth.expert(4096, 2048, 8, "cuda")
    for width in [2, 9, 26, 32]:
        x = synth.activations(width, 4096, 90 + width, "cuda")
        a = H(rt.expert_forward(x, g, u, d).output)
        b = H(rt_unfused.expert_forward(x, g, u, d).output)
        assert np.array_equal(a, b), f"width {width}"


# ----------------------------------------------------------------- router
@pytest.mark.parametrize("tokens", [1, 8, 128])
def test_route_bit_exact_vs_oracle(rt, tokens):
    from mimo_prismwing_b200 import synth
    w, bias = synth.router(256, 4096, 5, "cuda")
    x = synth.activations(tokens, 4096, 500 + tokens, "cuda")
    sel, wts, st = rt.route(x, w, bias)
    wbits = H(w.view(torch.int16)).view(np.uint16)
    logits = O.router_logits(H(x), wbits)
    osel, owts, _, margin, ties = O.noaux_topk(logits, H(bias))
    assert np.array_equal(H(sel).astype(np.uint32), osel)
    assert np.array_equal(H(wts).view(np.uint32), owts.view(np.uint32))
    assert st["boundary_tie_rows"] == ties


@pytest.mark.parametrize("tokens", [1, 8, 128])
def test_route_f32_weights_bit_exact_vs_oracle(rt, tokens):
    # The checkpoint's gate.weight is F32 (src/text_endpoint.rs:4350-4358,
    # f32_linear :3458): routed as F32, not through a bf16 copy.
    from mimo_prismwing_b200 import synth
    w, bias = synth.router_f32(256, 4096, 15, "cuda")
    wn = H(w)
    assert np.mean((wn.view(np.uint32) & 0xFFFF) != 0) > 0.99  # bits bf16 cannot hold
    x = synth.activations(tokens, 4096, 510 + tokens, "cuda")
    sel, wts, st = rt.route(x, w, bias)
    logits = O.router_logits(H(x), wn)
    osel, owts, _, _, ties = O.noaux_topk(logits, H(bias))
    assert np.array_equal(H(sel).astype(np.uint32), osel)
    assert np.array_equal(H(wts).view(np.uint32), owts.view(np.uint32))
    assert st["boundary_tie_rows"] == ties
    # a bf16 copy of the same weights is a different router
    wb = H(w.to(torch.bfloat16).view(torch.int16)).view(np.uint16)
    assert not np.array_equal(O.router_logits(H(x), wb), logits)


def test_moe_layer_f32_router_vs_oracle(rt):
    from gpu_helpers import assert_close_bf16, bank_arrays
    from mimo_prismwing_b200 import synth
    E, Hd, I, T = 64, 1024, 512, 8
    bank = _small_bank(E, Hd, I, 19)
    handle = rt.create_bank(bank)
    w, bias = synth.router_f32(E, Hd, 20, "cuda")
    x = synth.activations(T, Hd, 21, "cuda")
    ex = rt.moe_layer(x, w, bias, handle, want_routes=True)
    osel, owts, _, _, _ = O.noaux_topk(O.router_logits(H(x), H(w)), H(bias))
    assert np.array_equal(H(ex.selected).astype(np.uint32), osel)
    assert np.array_equal(H(ex.weights).view(np.uint32), owts.view(np.uint32))
    ref = O.routed_layer(H(x), osel, owts, bank_arrays(bank), O.ACC_F64, O.EXP_SLEEF)
    assert_close_bf16(H(ex.output), ref, what="moe layer f32 router")


def test_route_rejects_bad_weight_dtype(rt):
    import ctypes
    from mimo_prismwing_b200 import synth
    from mimo_prismwing_b200.runtime import PrismwingError
    w, bias = synth.router_f32(16, 512, 22, "cuda")
    r = rt._router(w, bias)
    r.weight_dtype = 7
    x = torch.zeros((1, 512), device="cuda")
    sel = torch.empty((1, 8), dtype=torch.int32, device="cuda")
    wts = torch.empty((1, 8), device="cuda")
    st = rt._L.pw_route(rt._rt, ctypes.byref(r), ctypes.c_void_p(x.data_ptr()), 1, ctypes.c_void_p(sel.data_ptr()),
                        ctypes.c_void_p(wts.data_ptr()), 0, None)
    assert st == -1 and "weight_dtype" in rt.last_error()
    with pytest.raises(PrismwingError):
        rt.route(x, w.half(), bias)


def test_route_host_io_matches_device_io(rt):
    from mimo_prismwing_b200 import synth
    w, bias = synth.router(256, 4096, 6, "cuda")
    x = synth.activations(8, 4096, 600, "cuda")
    a = rt.route(x, w, bias)
    b = rt.route(x.cpu(), w, bias)
    assert np.array_equal(H(a[0]), H(b[0])) and np.array_equal(H(a[1]), H(b[1]))


# ------------------------------------------------------------ routed layer
def _small_bank(n, hidden, inter, seed):
    from mimo_prismwing_b200 import synth
    return [synth.expert(hidden, inter, seed * 1000 + e, "cuda") for e in range(n)]


def test_moe_execute_host_schedule_vs_oracle(rt):
    # WideMetalMoeRuntime::execute with a BTreeMap-style schedule (8 tokens, 24 experts)
    from gpu_helpers import assert_close_bf16, bank_arrays
    from mimo_prismwing_b200 import synth
    from mimo_prismwing_b200.runtime import WideExpertBinding
    E, Hd, I, T = 24, 4096, 2048, 8
    bank = _small_bank(E, Hd, I, 3)
    rng = np.random.default_rng(3)
    sel = np.stack([rng.choice(E, 8, replace=False) for _ in range(T)]).astype(np.uint32)
    raw = rng.random((T, 8)).astype(np.float32)
    wts = (raw / raw.sum(1, keepdims=True)).astype(np.float32)
    x = synth.activations(T, Hd, 33, "cuda")
    offsets, order = O.schedule(sel, E)
    bindings = []
    for e in range(E):
        pl = order[offsets[e]:offsets[e + 1]]
        if len(pl) == 0:
            continue
        g, u, d = bank[e]
        bindings.append(WideExpertBinding(e, [int(p) // 8 for p in pl], [float(wts.ravel()[p]) for p in pl], g, u, d))
    ex = rt.execute_fused_gate_up(x, bindings)
    ref = O.routed_layer(H(x), sel, wts, bank_arrays(bank), O.ACC_F64, O.EXP_SLEEF)
    assert_close_bf16(H(ex.output), ref, what="moe execute")
    assert ex.expert_rows == T * 8 and ex.unique_experts == len(bindings)


def test_moe_execute_rejects_bad_schedule(rt):
    from mimo_prismwing_b200.runtime import PrismwingError, WideExpertBinding
    bank = _small_bank(1, 256, 256, 4)
    g, u, d = bank[0]
    x = torch.zeros((1, 256), device="cuda")
    with pytest.raises(PrismwingError) as e:  # 7 placements for one row
        rt.execute(x, [WideExpertBinding(0, [0] * 7, [0.125] * 7, g, u, d)])
    assert e.value.kind == "schedule"
    with pytest.raises(PrismwingError) as e:  # position out of range
        rt.execute(x, [WideExpertBinding(0, [0] * 7 + [1], [0.125] * 8, g, u, d)])
    assert e.value.kind == "schedule"


# token counts on both sides of the decode fusion: below 64 tokens the
# router's logits kernel also quantizes the activations
@pytest.mark.parametrize("tokens,E,Hd,I", [(8, 256, 4096, 2048), (1, 64, 1024, 512), (32, 64, 1024, 512),
                                           (40, 32, 512, 256), (63, 64, 1024, 512), (64, 64, 1024, 512)])
def test_moe_layer_device_router_vs_oracle(rt, tokens, E, Hd, I):
    from gpu_helpers import assert_close_bf16, bank_arrays
    from mimo_prismwing_b200 import synth
    bank = _small_bank(E, Hd, I, 9)
    handle = rt.create_bank(bank)
    w, bias = synth.router(E, Hd, 10, "cuda")
    x = synth.activations(tokens, Hd, 11, "cuda")
    ex = rt.moe_layer(x, w, bias, handle, want_routes=True)
    logits = O.router_logits(H(x), H(w.view(torch.int16)).view(np.uint16))
    osel, owts, _, _, _ = O.noaux_topk(logits, H(bias))
    assert np.array_equal(H(ex.selected).astype(np.uint32), osel)
    assert np.array_equal(H(ex.weights).view(np.uint32), owts.view(np.uint32))
    ref = O.routed_layer(H(x), osel, owts, bank_arrays(bank), O.ACC_F64, O.EXP_SLEEF)
    assert_close_bf16(H(ex.output), ref, what=f"moe layer T{tokens} E{E}")
    assert ex.expert_rows == tokens * 8
    assert ex.unique_experts == len(set(osel.ravel().tolist()))
    # host I/O
    ex2 = rt.moe_layer(x.cpu(), w, bias, handle)
    assert np.array_equal(ex2.output.numpy(), H(ex.output))


@pytest.mark.parametrize("tokens", [1, 8])
def test_moe_layer_equals_host_schedule_bitwise(rt, tokens):
    # The device-routed decode layer (device router, schedule and groups) and
    # the host-scheduled execute (src/wide_metal_moe.rs:836) over the same
    # routes run the same GEMVs and combine order: bit-identical outputs.
    from mimo_prismwing_b200 import synth
    from mimo_prismwing_b200.runtime import WideExpertBinding
    E, Hd, I = 256, 4096, 2048
    bank = _small_bank(E, Hd, I, 12)
    handle = rt.create_bank(bank)
    w, bias = synth.router(E, Hd, 13, "cuda")
    x = synth.activations(tokens, Hd, 14 + tokens, "cuda")
    ex = rt.moe_layer(x, w, bias, handle, want_routes=True)
    sel = H(ex.selected).astype(np.uint32)
    wts = H(ex.weights)
    offsets, order = O.schedule(sel, E)
    bindings = []
    for e in range(E):
        pl = order[offsets[e]:offsets[e + 1]]
        if len(pl):
            g, u, d = bank[e]
            bindings.append(WideExpertBinding(e, [int(p) // 8 for p in pl], [float(wts.ravel()[p]) for p in pl],
                                              g, u, d))
    ref = rt.execute_fused_gate_up(x, bindings)
    assert np.array_equal(H(ex.output), H(ref.output))


def test_bank_rejects_nonfinite_weight_byte(rt):
    from mimo_prismwing_b200.runtime import PrismwingError
    bank = _small_bank(9, 256, 256, 12)
    bank[4][1].weight[17, 5] = 0x7F
    with pytest.raises(PrismwingError) as e:
        rt.create_bank(bank)
    assert e.value.kind == "nonfinite" and "4" in str(e.value)


def test_repeated_calls_are_graph_capturable(rt):
    # After a first call of a shape (which uploads its launch descriptors),
    # asynchronous projection and expert calls enqueue only kernels: captured
    # into a CUDA graph and replayed they give the same bits as direct calls.
    from mimo_prismwing_b200 import synth
    s = torch.cuda.Stream()
    rt.set_stream(s)
    try:
        b = synth.projection(2048, 4096, 81, "cuda")
        g, u, d = synth.expert(4096, 2048, 82, "cuda")
        x1 = synth.activations(1, 4096, 83, "cuda")
        x8 = synth.activations(8, 4096, 84, "cuda")
        ref_gemv = rt.fp8_gemv(x1, b).output.clone()
        ref_lin = rt.execute_fp8_linear(x8, b).output.clone()
        ref_exp = rt.expert_forward(x8, g, u, d).output.clone()
        y_gemv = torch.empty_like(ref_gemv)
        y_lin = torch.empty_like(ref_lin)
        y_exp = torch.empty_like(ref_exp)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            rt.fp8_gemv(x1, b, asynchronous=True, out=y_gemv)
            rt.execute_fp8_linear(x8, b, asynchronous=True, out=y_lin)
            rt.expert_forward(x8, g, u, d, asynchronous=True, out=y_exp)
        for _ in range(3):
            with torch.cuda.stream(s):
                graph.replay()
            s.synchronize()
            assert torch.equal(y_gemv, ref_gemv) and torch.equal(y_lin, ref_lin) and torch.equal(y_exp, ref_exp)
        assert rt.error_flags() == 0
        del graph
    finally:
        rt.set_stream(None)


def test_first_call_of_a_shape_inside_capture_is_refused(rt):
    from mimo_prismwing_b200 import synth
    from mimo_prismwing_b200.runtime import PrismwingError
    s = torch.cuda.Stream()
    rt.set_stream(s)
    try:
        b = synth.projection(256, 512, 85, "cuda")
        x = synth.activations(3, 512, 86, "cuda")
        y = torch.empty((3, 256), device="cuda")
        graph = torch.cuda.CUDAGraph()
        with pytest.raises(PrismwingError) as e:
            with torch.cuda.graph(graph, stream=s):
                rt.execute_fp8_linear(x, b, asynchronous=True, out=y)
        assert "before capturing" in str(e.value)
    finally:
        rt.set_stream(None)
