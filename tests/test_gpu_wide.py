"""GPU parity of the wide (prefill) path: the tcgen05 grouped GEMM.

Widths >= 32 for projections and experts, expert groups of more than 16
placements in a host-built schedule, and routed layers of >= 256 tokens run
on the tcgen05/TMEM grouped GEMM instead of the GEMV.  Same oracle and
tolerances as the narrow path.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


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


@pytest.mark.parametrize("rows,cols,width", [(2048, 4096, 32), (2048, 4096, 100), (4096, 2048, 256),
                                             (256, 384, 40), (1024, 4096, 2048)])
def test_wide_linear_vs_oracle(rt, rows, cols, width):
    from gpu_helpers import assert_close, assert_close_bf16
    from mimo_prismwing_b200 import synth
    b = synth.projection(rows, cols, rows * 7 + cols, "cuda")
    x = synth.activations(width, cols, width + 3, "cuda")
    y32 = H(rt.execute_fp8_linear(x, b, f32_output=True).output)
    codes, scales, _ = O.dynamic_fp8(H(x))
    take = slice(None) if width <= 256 else slice(0, width, 7)  # keep the f64 oracle quick
    pre = O.blockscaled_linear(H(b.weight), H(b.scale), codes[take], scales[take])
    assert_close(y32[take], pre, what=f"wide linear {rows}x{cols} w{width}")
    y = H(rt.execute_fp8_linear(x, b).output)
    assert np.array_equal(O.round_bf16(y32), y)
    assert_close_bf16(y[take], O.round_bf16(pre), what=f"wide linear bf16 w{width}")


@pytest.mark.parametrize("width", [32, 64, 130])
def test_wide_expert_vs_oracle(rt, width):
    from gpu_helpers import assert_close_bf16, bank_arrays
    from mimo_prismwing_b200 import synth
    g, u, d = synth.expert(4096, 2048, 17, "cuda")
    x = synth.activations(width, 4096, 170 + width, "cuda")
    y = H(rt.expert_forward(x, g, u, d).output)
    (gw, gs, uw, us, dw, ds), = bank_arrays([(g, u, d)])
    xc, xs, _ = O.dynamic_fp8(H(x))
    gate = O.blockscaled_linear(gw, gs, xc, xs)
    up = O.blockscaled_linear(uw, us, xc, xs)
    act = O.staged_swiglu(gate, up, O.EXP_SLEEF)
    hc, hs, _ = O.dynamic_fp8(act)
    ref = O.round_bf16(O.blockscaled_linear(dw, ds, hc, hs))
    assert_close_bf16(y, ref, what=f"wide expert w{width}")


def test_wide_fused_gate_up_is_exact_against_unfused(rt, rt_unfused):
    # src/wide_metal_moe.rs:1343 at widths that take the tcgen05 path
    from mimo_prismwing_b200 import synth
    g, u, d = synth.expert(1024, 512, 18, "cuda")
    for width in [32, 96]:
        x = synth.activations(width, 1024, 180 + width, "cuda")
        a = H(rt.expert_forward(x, g, u, d).output)
        b = H(rt_unfused.expert_forward(x, g, u, d).output)
        assert np.array_equal(a, b), f"width {width}"


def test_wide_fused_quantizer_exact_over_magnitudes(rt, rt_unfused):
    # The fused path quantizes the SwiGLU output with reciprocal-based
    # quotients; the unfused path divides (pw_quantize semantics).  Token rows
    # scaled by 2^-40 .. 2^40 put the hidden values and their group scales
    # across ~80 binades; every hidden code, hence every down row, must match.
    from mimo_prismwing_b200 import synth
    g, u, d = synth.expert(2048, 1024, 23, "cuda")
    width = 512
    x = synth.activations(width, 2048, 77, "cuda")
    k = torch.arange(width, device="cuda", dtype=torch.float32)
    x = x * torch.exp2(torch.remainder(k * 37.0, 81.0) - 40.0).unsqueeze(1)
    a = H(rt.expert_forward(x, g, u, d).output)
    b = H(rt_unfused.expert_forward(x, g, u, d).output)
    assert np.array_equal(a, b)


def test_wide_host_schedule_vs_oracle(rt):
    # every token routed to all 8 experts: 64 placements per expert (> 16)
    from gpu_helpers import assert_close_bf16, bank_arrays
    from mimo_prismwing_b200 import synth
    from mimo_prismwing_b200.runtime import WideExpertBinding
    E, Hd, I, T = 8, 1024, 512, 64
    bank = [synth.expert(Hd, I, 300 + e, "cuda") for e in range(E)]
    rng = np.random.default_rng(5)
    sel = np.stack([rng.permutation(E) for _ in range(T)]).astype(np.uint32)
    raw = rng.random((T, 8)).astype(np.float32)
    wts = (raw / raw.sum(1, keepdims=True)).astype(np.float32)
    x = synth.activations(T, Hd, 301, "cuda")
    offsets, order = O.schedule(sel, E)
    bindings = []
    for e in range(E):
        pl = order[offsets[e]:offsets[e + 1]]
        g, u, d = bank[e]
        bindings.append(WideExpertBinding(e, [int(p) // 8 for p in pl], [float(wts.ravel()[p]) for p in pl], g, u, d))
    ex = rt.execute_fused_gate_up(x, bindings)
    ref = O.routed_layer(H(x), sel, wts, bank_arrays(bank), O.ACC_F64, O.EXP_SLEEF)
    assert_close_bf16(H(ex.output), ref, what="wide host schedule")


@pytest.mark.parametrize("tokens", [256, 512])
def test_wide_moe_layer_device_router_vs_oracle(rt, tokens):
    from gpu_helpers import assert_close_bf16, bank_arrays
    from mimo_prismwing_b200 import synth
    E, Hd, I = 32, 1024, 512
    bank = [synth.expert(Hd, I, 400 + e, "cuda") for e in range(E)]
    handle = rt.create_bank(bank)
    w, bias = synth.router(E, Hd, 41, "cuda")
    x = synth.activations(tokens, Hd, 42, "cuda")
    ex = rt.moe_layer(x, w, bias, handle, want_routes=True)
    logits = O.router_logits(H(x), H(w.view(torch.int16)).view(np.uint16))
    osel, owts, _, _, _ = O.noaux_topk(logits, H(bias))
    assert np.array_equal(H(ex.selected).astype(np.uint32), osel)
    ref = O.routed_layer(H(x), osel, owts, bank_arrays(bank), O.ACC_F64, O.EXP_SLEEF)
    assert_close_bf16(H(ex.output), ref, what=f"wide moe layer T{tokens}")
    assert ex.expert_rows == tokens * 8


def test_full_size_prefill_layer_vs_oracle(rt):
    # The benchmarked layer itself (one layer): 2048
    # tokens, 256 experts of [2048x4096] gate/up and [4096x2048] down, device
    # router (src/text_endpoint.rs:5076-5103 gate the reference's layer-major
    # slices the same way).  Routes and route weights are compared bit for bit
    # on every token; the output against the f64 oracle on every 16th token
    # (each token's output depends only on its own row and routes).
    from gpu_helpers import assert_close_bf16
    from mimo_prismwing_b200 import synth
    E, Hd, I, T = 256, 4096, 2048, 2048
    bank = [synth.expert(Hd, I, 9000 + e, "cuda") for e in range(E)]
    handle = rt.create_bank(bank)
    w, bias = synth.router(E, Hd, 77, "cuda")
    x = synth.activations(T, Hd, 78, "cuda")
    ex = rt.moe_layer(x, w, bias, handle, want_routes=True)
    logits = O.router_logits(H(x), H(w.view(torch.int16)).view(np.uint16))
    osel, owts, _, _, _ = O.noaux_topk(logits, H(bias))
    assert np.array_equal(H(ex.selected).astype(np.uint32), osel)
    assert np.array_equal(H(ex.weights).view(np.uint32), owts.view(np.uint32))
    assert ex.expert_rows == T * 8 and ex.unique_experts == E
    take = np.arange(0, T, 16)
    needed = sorted(set(osel[take].ravel().tolist()))
    arrays = {e: tuple(H(t) for p in bank[e] for t in (p.weight, p.scale)) for e in needed}
    filler = arrays[needed[0]]
    oracle_bank = [arrays.get(e, filler) for e in range(E)]  # the oracle reads only selected experts
    ref = O.routed_layer(H(x)[take], osel[take], owts[take], oracle_bank, O.ACC_F64, O.EXP_SLEEF)
    assert_close_bf16(H(ex.output)[take], ref, what="configs[4] layer (every 16th token)")
    # the asynchronous device call gives the same bits
    out = torch.empty_like(x)
    rt.moe_layer(x, w, bias, handle, asynchronous=True, out=out)
    rt.synchronize()
    assert torch.equal(out, ex.output)


@pytest.mark.parametrize("experts,hidden,tokens,dtype", [(256, 4096, 64, "bf16"), (256, 4096, 67, "bf16"),
                                                         (100, 1024, 70, "bf16"), (256, 4096, 2048, "bf16"),
                                                         (256, 4096, 67, "f32"), (256, 4096, 2048, "f32")])
def test_wide_route_bit_exact_vs_oracle(rt, experts, hidden, tokens, dtype):
    # >= 64 tokens take the register-tiled router (64 tokens x 128 experts x
    # one 256-column slice per unit); ragged token and expert tiles included;
    # F32 weights are the checkpoint's gate.weight (src/text_endpoint.rs:4350)
    from mimo_prismwing_b200 import synth
    make = synth.router_f32 if dtype == "f32" else synth.router
    w, bias = make(experts, hidden, 51, "cuda")
    x = synth.activations(tokens, hidden, 700 + tokens, "cuda")
    sel, wts, st = rt.route(x, w, bias)
    logits = O.router_logits(H(x), H(w) if dtype == "f32" else H(w.view(torch.int16)).view(np.uint16))
    osel, owts, _, _, ties = O.noaux_topk(logits, H(bias))
    assert np.array_equal(H(sel).astype(np.uint32), osel)
    assert np.array_equal(H(wts).view(np.uint32), owts.view(np.uint32))
    assert st["boundary_tie_rows"] == ties


@pytest.mark.parametrize("layout,width", [("full", 64), ("full", 2048), ("swa", 40), ("swa", 300)])
def test_wide_qkv_layouts_vs_oracle(rt, layout, width):
    # the fused QKV projection with its per-segment scale grid on
    # the tcgen05 GEMM (each 128-row tile = two 64-row checkpoint runs)
    from gpu_helpers import assert_close, assert_close_bf16
    from mimo_prismwing_b200 import synth
    b = synth.full_qkv(31, "cuda") if layout == "full" else synth.swa_qkv(32, "cuda")
    lay = O.LAYOUT_FULL_QKV if layout == "full" else O.LAYOUT_SWA_QKV
    x = synth.activations(width, 4096, 60 + width, "cuda")
    full = layout == "full"
    y32 = H(rt.execute_fp8_linear(x, b, full_qkv_layout=full, f32_output=True).output)
    codes, scales, _ = O.dynamic_fp8(H(x))
    take = slice(None) if width <= 300 else slice(0, width, 29)  # keep the f64 oracle quick
    ref = O.blockscaled_linear(H(b.weight), H(b.scale), codes[take], scales[take], layout=lay)
    assert_close(y32[take], ref, what=f"{layout} qkv w{width}")
    y = H(rt.execute_fp8_linear(x, b, full_qkv_layout=full).output)
    assert np.array_equal(O.round_bf16(y32), y)
    assert_close_bf16(y[take], O.round_bf16(ref), what=f"{layout} qkv bf16 w{width}")
