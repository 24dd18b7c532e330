"""CPU restatement of the reference's own torch implementation of the routed layer.

TEST INFRASTRUCTURE AND CPU BASELINE ONLY: bench.py's cpu_baseline and
--impl reference legs time it on the host cores; the product path never
imports it.

The reference generates its layer-major MoE authorities with torch on the CPU
(tools/generate_layer_major_moe_reference.py): `dequantize` (:72) widens the
e4m3 weight and multiplies by its 128x128 scale grid, `dynamic_input` (:84)
quantizes and dequantizes the activation per 128-column group, `bf16_widen`
(:97) is the bf16 staging point, and the layer loop (:194-239) runs, per
expert in ascending id, q @ gate.T, q @ up.T (f32 SGEMM), the staged SwiGLU,
the hidden's dynamic quantization, @ down.T, then index_add_ of the weighted
rows and a final bf16 round.  The same SGEMM formulation is the reference's
CPU "source" mode for a projection (fp8_linear, src/text_endpoint.rs:3053).
The router is route_mlp's f32 linear (src/text_endpoint.rs:4350-4358) as an
SGEMM, sigmoid, top-8 of score + bias and renormalised weights
(pytorch_noaux_routes :4394).

This is the fast CPU formulation (all host threads through torch's SGEMM);
oracle/pw_oracle.c is the bit-level restatement the parity tests use.
"""
from __future__ import annotations

import torch

TOP_K = 8


def set_threads(n: int) -> None:
    torch.set_num_threads(max(1, int(n)))


def dequantize(weight_u8: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """tools/generate_layer_major_moe_reference.py:72: e4m3 -> f32, times the block scale."""
    w = weight_u8.view(torch.float8_e4m3fn).float()
    return w * scale.repeat_interleave(128, 0)[: w.shape[0]].repeat_interleave(128, 1)


def dynamic_input(values: torch.Tensor) -> torch.Tensor:
    """tools/generate_layer_major_moe_reference.py:84: per-token, group-128 FP8 round trip."""
    rows, columns = values.shape
    grouped = values.float().reshape(rows, columns // 128, 128)
    scales = grouped.abs().amax(-1).clamp(min=1.0e-10) / 448.0
    encoded = torch.clamp(grouped / scales.unsqueeze(-1), -448.0, 448.0).to(torch.float8_e4m3fn)
    return (encoded.float() * scales.unsqueeze(-1)).reshape(rows, columns)


def bf16_widen(values: torch.Tensor) -> torch.Tensor:
    """tools/generate_layer_major_moe_reference.py:97: the bf16 staging point."""
    return values.to(torch.bfloat16).float()


def route(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor):
    """route_mlp (src/text_endpoint.rs:4342): f32 logits by SGEMM, sigmoid
    scores, top-8 of score + bias, weights = score / (sum + 1e-20)."""
    logits = x.float() @ weight.float().T
    scores = torch.sigmoid(logits)
    _, selected = torch.topk(scores + bias.float(), TOP_K, dim=-1)
    picked = scores.gather(1, selected)
    return selected, picked / (picked.sum(-1, keepdim=True) + 1.0e-20)


def expert_forward(values: torch.Tensor, gate, up, down) -> torch.Tensor:
    """One expert (tools/generate_layer_major_moe_reference.py:194-211): each of
    gate/up/down is a (weight u8, scale f32) pair; returns bf16-valued rows."""
    g = dequantize(*gate)
    u = dequantize(*up)
    d = dequantize(*down)
    q = dynamic_input(values)
    gate_values = bf16_widen(q @ g.T)
    up_values = bf16_widen(q @ u.T)
    silu_values = bf16_widen(gate_values / (1.0 + torch.exp(-gate_values)))
    activated = bf16_widen(silu_values * up_values)
    return bf16_widen(dynamic_input(activated) @ d.T)


def routed_layer(x: torch.Tensor, selected: torch.Tensor, weights: torch.Tensor, bank, experts=None,
                 finish: bool = True) -> torch.Tensor:
    """The layer loop (tools/generate_layer_major_moe_reference.py:180-239):
    experts in ascending id, index_add_ of route-weighted rows, final bf16
    round.  bank[e] = ((gate_w, gate_s), (up_w, up_s), (down_w, down_s)) CPU
    tensors.  `experts` (optional) restricts the loop to those ids, for timed
    samples of a layer; `finish=False` skips the final bf16 round."""
    tokens, hidden = x.shape
    output = torch.zeros((tokens, hidden), dtype=torch.float32)
    flat_sel = selected.reshape(-1)
    flat_w = weights.reshape(-1).float()
    order = torch.argsort(flat_sel, stable=True)
    ids, counts = torch.unique_consecutive(flat_sel[order], return_counts=True)
    begin = 0
    wanted = None if experts is None else set(int(e) for e in experts)
    for e, n in zip(ids.tolist(), counts.tolist()):
        placements = order[begin:begin + n]
        begin += n
        if wanted is not None and e not in wanted:
            continue
        positions = placements // TOP_K
        projected = expert_forward(x[positions], *bank[e])
        output.index_add_(0, positions, projected * flat_w[placements].unsqueeze(1))
    return bf16_widen(output) if finish else output
