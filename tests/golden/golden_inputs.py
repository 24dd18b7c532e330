"""Seeded inputs for the torch-reference expert goldens (tests/golden/).

The weights are regenerated from their seed wherever the goldens are checked,
so only the reference's outputs are stored.  numpy's PCG64 stream and torch's
CPU float8_e4m3fn cast (round-to-nearest-even) are both deterministic, so the
same bytes come out on every machine with this image.
"""
from __future__ import annotations

import base64

import numpy as np
import torch


def quantize_block_fp8(w: np.ndarray):
    """Per 128x128 block: scale = amax/448, codes = RNE e4m3(w/scale)."""
    rows, cols = w.shape
    t = torch.from_numpy(np.ascontiguousarray(w, dtype=np.float32))
    blocks = t.reshape(rows // 128, 128, cols // 128, 128)
    amax = blocks.abs().amax(dim=(1, 3)).clamp(min=1e-12)
    scale = (amax / 448.0).float()
    q = (blocks / scale[:, None, :, None]).to(torch.float8_e4m3fn)
    return q.reshape(rows, cols).view(torch.uint8).numpy().copy(), scale.numpy().copy()


def expert_case(seed: int, hidden: int, inter: int, width: int):
    rng = np.random.default_rng(seed)
    gw, gs = quantize_block_fp8(rng.normal(0.0, 0.02, (inter, hidden)).astype(np.float32))
    uw, us = quantize_block_fp8(rng.normal(0.0, 0.02, (inter, hidden)).astype(np.float32))
    dw, ds = quantize_block_fp8(rng.normal(0.0, 0.02, (hidden, inter)).astype(np.float32))
    x = rng.normal(0.0, 1.0, (width, hidden)).astype(np.float32)
    x = torch.from_numpy(x).to(torch.bfloat16).float().numpy().copy()
    return {"x": x, "gate_w": gw, "gate_s": gs, "up_w": uw, "up_s": us, "down_w": dw, "down_s": ds}


def pack_f32(a) -> str:
    return base64.b64encode(np.ascontiguousarray(a, dtype="<f4").tobytes()).decode()


def unpack_f32(s: str, shape) -> np.ndarray:
    return np.frombuffer(base64.b64decode(s), dtype="<f4").reshape(shape).copy()
