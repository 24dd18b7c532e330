"""GPU parity of the steps either side of the routed layer.

Before it: the decoder layer's post-attention RMSNorm (src/text_endpoint.rs:2939
rms_norm, PyTorch's cascade order for the sum of squares, pinned by the
reference's pw0079 fixture), bit-exact.  After it: the residual add
bf16(post_attention + mlp) (src/text_endpoint.rs:5576-5580).  pw_moe_block
fuses both around the routed layer; it must equal the composition of the
separate calls bit for bit, and the oracle within the layer tolerance.
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


def H(t):
    from gpu_helpers import host
    return host(t)


def _bf16_weight(n, seed):
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return (1.0 + 0.1 * torch.randn(n, generator=g)).to(torch.bfloat16)


def test_rms_norm_matches_pytorch_cascade_fixture(rt):
    # src/lib.rs:7917: a real post-attention row; the GPU's inverse RMS has the
    # fixture's bits (PyTorch's cascade order, not a high-precision sum)
    with open(os.path.join(GOLDEN, "pw0079_rms_cascade.json")) as f:
        fx = json.load(f)
    x = (np.asarray(fx["input_bf16_u16"], dtype=np.uint32) << 16).view(np.float32).reshape(1, -1)
    eps = float(np.uint32(fx["epsilon_f32_u32"]).view(np.float32))
    w = _bf16_weight(4096, 3)
    y, inv = rt.rms_norm(torch.from_numpy(x).cuda(), w.cuda(), eps)
    assert int(H(inv).view(np.uint32)[0]) == fx["inverse_f32_u32"]
    ref, _ = O.rms_norm(x, w.float().numpy(), eps)
    assert np.array_equal(H(y).view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("rows,cols,dtype", [(1, 4096, "bf16"), (37, 4096, "f32"), (5, 256, "bf16"),
                                             (3, 16384, "f32"), (2048, 4096, "bf16"), (4, 1280, "bf16")])
def test_rms_norm_bit_exact_vs_oracle(rt, rows, cols, dtype):
    rng = np.random.default_rng(rows * 7 + cols)
    x = O.round_bf16((rng.standard_normal((rows, cols)) * rng.uniform(0.01, 30.0, (rows, 1))).astype(np.float32))
    x[0, :7] = [0.0, -0.0, 1e-30, -3.5, 65504.0, 1e-8, -0.25]
    w = _bf16_weight(cols, cols)
    wt = w.float() if dtype == "f32" else w
    y, inv = rt.rms_norm(torch.from_numpy(x).cuda(), wt.cuda(), 1e-5)
    ref, rinv = O.rms_norm(x, w.float().numpy(), 1e-5)
    assert np.array_equal(H(inv).view(np.uint32), rinv.view(np.uint32))
    assert np.array_equal(H(y).view(np.uint32), ref.view(np.uint32))
    # host I/O gives the same bits
    yh, _ = rt.rms_norm(torch.from_numpy(x), wt.cuda(), 1e-5)
    assert np.array_equal(yh.numpy().view(np.uint32), ref.view(np.uint32))


def test_rms_norm_rejects_bad_input(rt):
    from mimo_prismwing_b200.runtime import PrismwingError
    w = _bf16_weight(256, 1).cuda()
    x = torch.ones((2, 256), device="cuda")
    x[1, 17] = float("inf")
    with pytest.raises(PrismwingError) as e:
        rt.rms_norm(x, w, 1e-5)
    assert e.value.kind == "nonfinite"
    with pytest.raises(PrismwingError) as e:
        rt.rms_norm(torch.ones((1, 256), device="cuda"), w, 0.0)
    assert e.value.kind == "argument"
    with pytest.raises(PrismwingError) as e:
        rt.rms_norm(torch.ones((1, 384), device="cuda"), _bf16_weight(384, 2).cuda(), 1e-5)
    assert e.value.kind == "shape"


@pytest.mark.parametrize("tokens,E,Hd,I", [(8, 64, 1024, 512), (300, 32, 1024, 512)])
def test_moe_block_equals_norm_layer_residual_composition(rt, tokens, E, Hd, I):
    # pw_moe_block == bf16(residual + pw_moe_layer(pw_rms_norm(residual))), bit
    # for bit, on the GEMV (8 tokens) and tcgen05 (300 tokens) paths; and the
    # oracle's rms_norm -> routed layer -> residual add within the layer tolerance
    from gpu_helpers import assert_close_bf16, bank_arrays
    from mimo_prismwing_b200 import synth
    bank = [synth.expert(Hd, I, 5000 + 13 * tokens + e, "cuda") for e in range(E)]
    handle = rt.create_bank(bank)
    w, bias = synth.router_f32(E, Hd, 61, "cuda")
    rng = np.random.default_rng(tokens)
    resid = torch.from_numpy(O.round_bf16((rng.standard_normal((tokens, Hd)) * 4.0).astype(np.float32))).cuda()
    nw = _bf16_weight(Hd, 9).cuda()
    blk = rt.moe_block(resid, nw, 1e-5, w, bias, handle, want_routes=True)
    xn, _ = rt.rms_norm(resid, nw, 1e-5)
    lay = rt.moe_layer(xn, w, bias, handle, want_routes=True)
    assert torch.equal(blk.selected, lay.selected) and torch.equal(blk.weights, lay.weights)
    composed = O.residual_add(H(resid), H(lay.output))
    assert np.array_equal(H(blk.output).view(np.uint32), composed.view(np.uint32))
    # oracle
    xo, _ = O.rms_norm(H(resid), nw.float().cpu().numpy(), 1e-5)
    osel, owts, _, _, _ = O.noaux_topk(O.router_logits(xo, H(w)), H(bias))
    assert np.array_equal(H(blk.selected).astype(np.uint32), osel)
    mlp = O.routed_layer(xo, osel, owts, bank_arrays(bank), O.ACC_F64, O.EXP_SLEEF)
    assert_close_bf16(H(lay.output), mlp, what=f"block mlp T{tokens}")
    assert_close_bf16(H(blk.output), O.residual_add(H(resid), mlp), what=f"block T{tokens}")
    # host I/O and the asynchronous device call give the same bits
    hb = rt.moe_block(resid.cpu(), nw, 1e-5, w, bias, handle)
    assert np.array_equal(hb.output.numpy(), H(blk.output))
    out = torch.empty_like(resid)
    rt.moe_block(resid, nw, 1e-5, w, bias, handle, asynchronous=True, out=out)
    rt.synchronize()
    assert torch.equal(out, blk.output)


def test_moe_block_rejects_aliasing_and_bad_norm(rt):
    from mimo_prismwing_b200 import synth
    from mimo_prismwing_b200.runtime import PrismwingError
    bank = [synth.expert(512, 256, 70 + e, "cuda") for e in range(16)]
    handle = rt.create_bank(bank)
    w, bias = synth.router(16, 512, 62, "cuda")
    x = torch.ones((2, 512), device="cuda")
    with pytest.raises(PrismwingError) as e:  # output aliases the residual
        rt.moe_block(x, _bf16_weight(512, 1).cuda(), 1e-5, w, bias, handle, out=x)
    assert e.value.kind == "argument"
    with pytest.raises(PrismwingError) as e:  # norm width differs from the bank's hidden size
        rt.moe_block(x, _bf16_weight(256, 1).cuda(), 1e-5, w, bias, handle)
    assert e.value.kind == "shape"
    with pytest.raises(PrismwingError) as e:  # epsilon must be positive
        rt.moe_block(x, _bf16_weight(512, 1).cuda(), -1.0, w, bias, handle)
    assert e.value.kind == "argument"


@pytest.mark.parametrize("width", [1, 8, 40])
def test_dense_mlp_layer0_shape_vs_oracle(rt, width):
    # dense_mlp (src/text_endpoint.rs:4266): gate/up [16384, 4096], staged
    # SwiGLU, down [4096, 16384]; widths 1 and 8 on the GEMV, 40 on the
    # tcgen05 GEMM; the 16384-wide down projection runs in 4096-column slices
    from gpu_helpers import assert_close_bf16, bank_arrays
    from mimo_prismwing_b200 import synth
    g, u, d = synth.expert(4096, 16384, 44, "cuda")
    x = synth.activations(width, 4096, 90 + width, "cuda")
    ex = rt.dense_mlp(x, g, u, d)
    y = H(ex.output)
    (gw, gs, uw, us, dw, ds), = bank_arrays([(g, u, d)])
    take = slice(None) if width <= 8 else slice(0, width, 5)  # keep the f64 oracle quick
    xc, xs, _ = O.dynamic_fp8(H(x)[take])
    act = O.staged_swiglu(O.blockscaled_linear(gw, gs, xc, xs), O.blockscaled_linear(uw, us, xc, xs), O.EXP_SLEEF)
    hc, hs, _ = O.dynamic_fp8(act)
    ref = O.round_bf16(O.blockscaled_linear(dw, ds, hc, hs))
    assert_close_bf16(y[take], ref, what=f"dense MLP w{width}")
    assert ex.weight_bytes == 3 * 16384 * 4096 + 4 * (2 * 128 * 32 + 32 * 128)
    # host I/O: same bits
    assert np.array_equal(rt.dense_mlp(x.cpu(), g, u, d).output.numpy(), y)


def test_dense_mlp_small_intermediate_equals_expert_forward(rt):
    # at I <= 4096 the dense MLP is the routed expert's chain exactly
    from mimo_prismwing_b200 import synth
    g, u, d = synth.expert(1024, 2048, 45, "cuda")
    x = synth.activations(5, 1024, 46, "cuda")
    assert torch.equal(rt.dense_mlp(x, g, u, d).output, rt.expert_forward(x, g, u, d).output)
