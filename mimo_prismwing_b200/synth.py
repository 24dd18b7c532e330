"""Seeded synthetic inputs with the shapes and distributions of the benchmark configs.

Weights are drawn N(0, 0.02), each 128x128 block gets scale = amax/448 and the
codes are the round-to-nearest-even e4m3 of w/scale (torch's float8_e4m3fn
cast); activations are N(0, 1) rounded to bf16 values; the router weight is
bf16 N(0, 0.02) with an f32 correction bias N(0, 0.01).  There is no network
here for the MiMo-V2.5 checkpoint, so these stand in for its tensors.
"""
from __future__ import annotations

from typing import List, Tuple

import torch

from .runtime import WideProjectionBinding


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def quantize_blocks(w: torch.Tensor, row_blocks: List[Tuple[int, int]] | None = None):
    """Per-block FP8 quantization.  row_blocks lists the (start, end) source
    rows of each scale row (default: uniform 128-row blocks)."""
    rows, cols = w.shape
    if row_blocks is None:
        row_blocks = [(r, min(r + 128, rows)) for r in range(0, rows, 128)]
    kb = cols // 128
    scales = torch.empty((len(row_blocks), kb), dtype=torch.float32, device=w.device)
    codes = torch.empty((rows, cols), dtype=torch.uint8, device=w.device)
    for i, (a, b) in enumerate(row_blocks):
        blk = w[a:b].reshape(b - a, kb, 128)
        amax = blk.abs().amax(dim=(0, 2)).clamp(min=1e-12)
        s = (amax / 448.0).float()
        scales[i] = s
        q = (blk / s[None, :, None]).to(torch.float8_e4m3fn)
        codes[a:b] = q.reshape(b - a, cols).view(torch.uint8)
    return codes, scales


def projection(rows: int, cols: int, seed: int, device="cuda", row_blocks=None) -> WideProjectionBinding:
    g = _gen(device, seed)
    w = torch.randn((rows, cols), generator=g, device=device, dtype=torch.float32) * 0.02
    codes, scales = quantize_blocks(w, row_blocks)
    return WideProjectionBinding(codes.contiguous(), scales.contiguous())


def activations(width: int, cols: int, seed: int, device="cuda") -> torch.Tensor:
    g = _gen(device, seed)
    x = torch.randn((width, cols), generator=g, device=device, dtype=torch.float32)
    return x.to(torch.bfloat16).float().contiguous()


def full_qkv_row_blocks() -> List[Tuple[int, int]]:
    """Source-row ranges of the 108 full-QKV scale rows: per shard of 3392
    rows, 24 Q blocks, a 128-row and a partial 64-row K block, one V block
    (src/text_endpoint.rs:3227 full_qkv_scale_row)."""
    out = []
    for shard in range(4):
        base = shard * 3392
        out += [(base + 128 * i, base + 128 * (i + 1)) for i in range(24)]
        out += [(base + 3072, base + 3200), (base + 3200, base + 3264), (base + 3264, base + 3392)]
    return out


def full_qkv(seed: int, device="cuda") -> WideProjectionBinding:
    return projection(13568, 4096, seed, device, full_qkv_row_blocks())


def swa_qkv(seed: int, device="cuda") -> WideProjectionBinding:
    return projection(14848, 4096, seed, device)


def expert(hidden: int, inter: int, seed: int, device="cuda"):
    return (projection(inter, hidden, seed * 3 + 0, device),
            projection(inter, hidden, seed * 3 + 1, device),
            projection(hidden, inter, seed * 3 + 2, device))


def router(experts: int, hidden: int, seed: int, device="cuda"):
    """bf16 router weight N(0, 0.02) and f32 bias N(0, 0.01)."""
    g = _gen(device, seed)
    w = (torch.randn((experts, hidden), generator=g, device=device) * 0.02).to(torch.bfloat16).contiguous()
    bias = (torch.randn((experts,), generator=g, device=device) * 0.01).float().contiguous()
    return w, bias


def router_f32(experts: int, hidden: int, seed: int, device="cuda"):
    """F32 router weight N(0, 0.02), as the checkpoint stores gate.weight
    (most values carry mantissa bits that bf16 cannot hold), and f32 bias."""
    g = _gen(device, seed)
    w = (torch.randn((experts, hidden), generator=g, device=device) * 0.02).float().contiguous()
    bias = (torch.randn((experts,), generator=g, device=device) * 0.01).float().contiguous()
    return w, bias


def to_device(obj, device):
    """Copy a tensor, a WideProjectionBinding, or a tuple/list of them, to `device`."""
    if isinstance(obj, torch.Tensor):
        return obj.to(device).contiguous()
    if isinstance(obj, WideProjectionBinding):
        return WideProjectionBinding(obj.weight.to(device).contiguous(), obj.scale.to(device).contiguous())
    return type(obj)(to_device(o, device) for o in obj)
