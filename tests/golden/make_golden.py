#!/usr/bin/env python3
"""Regenerate the golden vectors under tests/golden/ from the reference tree.

Run where the x3haloed/mimo-prismwing source is checked out (its location is
the --reference argument).  The GPU box never runs this script: the tests read
only the JSON files it writes.

Two kinds of golden data come out:
  * copies of the reference's own fixtures for the hot path (the files named in
    its tests: src/lib.rs:7966-8076, src/text_endpoint.rs:14035-14800), trimmed
    to the keys the tests use;
  * vectors produced by importing the reference's own torch implementation of
    the expert path (tools/generate_layer_major_moe_reference.py:53-98:
    build_schedule, dynamic_input, bf16_widen) on small seeded inputs.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

COPIES = {
    # out name: (reference fixture path, keys kept or None for all)
    "f8_e4m3fn_all_bytes.json": ("evals/fixtures/tiny/f8-e4m3fn-all-bytes.json", ["expected_f32_bits", "oracle"]),
    "pw0053_dynamic_fp8.json": ("evals/fixtures/tiny/pw0053-dynamic-fp8-activation.json", None),
    "pw0054_bf16_boundary.json": ("evals/fixtures/tiny/pw0054-bf16-boundary.json",
                                  ["input_f32_bits", "bf16_u16", "widened_f32_bits", "torch_version"]),
    "pw0062_router_sigmoid.json": ("evals/fixtures/tiny/pw0062-router-sigmoid.json", None),
    "pw0068_sleef_boundaries.json": ("evals/fixtures/tiny/pw0068-sleef-boundaries.json", None),
    "pw0063_topk_order.json": ("evals/fixtures/tiny/pw0063-topk-order.json", None),
    "pw0157_topk_ties.json": ("evals/fixtures/tiny/pw0157-pytorch-topk-ties.json",
                              ["cases", "standard_library", "top_k", "width"]),
    "swiglu_f32.json": ("evals/fixtures/tiny/swiglu-f32.json", None),
    "moe_noaux_tc_swiglu.json": ("evals/fixtures/tiny/moe-noaux-tc-swiglu.json", None),
    "mtp_gate_fp8_gemv.json": ("evals/fixtures/real/mtp-gate-fp8-gemv.json",
                               ["rows", "columns", "block_columns", "raw_u8", "scale_inv", "input",
                                "expected_f32", "oracle", "tensor"]),
    "pw0079_rms_cascade.json": ("evals/fixtures/tiny/pw0079-pytorch-rms-cascade.json",
                                ["epsilon_f32_u32", "high_precision_variance_f32_u32", "input_bf16_u16",
                                 "inverse_f32_u32", "semantic", "torch_version", "variance_f32_u32", "width"]),
    "mtp_gate_fp8_block.json": ("evals/fixtures/real/mtp-gate-fp8-block.json",
                                ["raw_u8", "decoded_fp8", "dequantized", "scale_inv"]),
}


def copy_fixtures(reference: str) -> None:
    for out, (src, keys) in COPIES.items():
        with open(os.path.join(reference, src)) as f:
            data = json.load(f)
        if keys is not None:
            data = {k: data[k] for k in keys if k in data}
        data["_source"] = src
        with open(os.path.join(HERE, out), "w") as f:
            json.dump(data, f, separators=(",", ":"))


def torch_expert_goldens(reference: str) -> None:
    """Small experts pushed through the reference's own torch helpers."""
    sys.path.insert(0, reference)
    import torch
    from tools.generate_layer_major_moe_reference import bf16_widen, build_schedule, dynamic_input

    sys.path.insert(0, HERE)
    from golden_inputs import expert_case, pack_f32

    cases = []
    for seed, hidden, inter, width in [(1, 256, 256, 1), (2, 256, 384, 3), (3, 512, 256, 8)]:
        c = expert_case(seed, hidden, inter, width)
        x = torch.from_numpy(c["x"])

        def deq(name):
            q = torch.from_numpy(c[name + "_w"]).view(torch.float8_e4m3fn).float()
            s = torch.from_numpy(c[name + "_s"])
            return q * s.repeat_interleave(128, 0).repeat_interleave(128, 1)

        # tools/generate_layer_major_moe_reference.py:196-205 (per-expert body)
        quantized = dynamic_input(x)
        gate = bf16_widen(quantized @ deq("gate").T)
        up = bf16_widen(quantized @ deq("up").T)
        silu = bf16_widen(gate / (1.0 + torch.exp(-gate)))
        act = bf16_widen(silu * up)
        projected = bf16_widen(dynamic_input(act) @ deq("down").T)
        cases.append({
            "seed": seed, "hidden": hidden, "intermediate": inter, "width": width,
            "gate": pack_f32(gate.numpy()), "up": pack_f32(up.numpy()),
            "act": pack_f32(act.numpy()), "down": pack_f32(projected.numpy()),
        })

    # tools/generate_layer_major_moe_reference.py:53 build_schedule on a seeded
    # 128-row route table (its ROWS/TOP_K constants).
    rng = np.random.default_rng(209)
    selected = np.stack([rng.choice(256, size=8, replace=False) for _ in range(128)]).astype(np.int64)
    raw = rng.random((128, 8)).astype(np.float32)
    weights = (raw / raw.sum(axis=1, keepdims=True)).astype(np.float32)
    schedule = build_schedule(selected, weights)
    sched = {str(k): v for k, v in sorted(schedule.items())}
    payload = {
        "_source": "tools/generate_layer_major_moe_reference.py (dynamic_input, bf16_widen, build_schedule)",
        "torch_version": torch.__version__,
        "experts": cases,
        "schedule_selected": selected.tolist(),
        "schedule_weights": weights.tolist(),
        "schedule": sched,
    }
    with open(os.path.join(HERE, "torch_reference_expert.json"), "w") as f:
        json.dump(payload, f, separators=(",", ":"))


def main() -> None:
    ap = argparse.ArgumentParser()
    env = os.environ.get("PW_REFERENCE_ROOT")
    ap.add_argument("--reference", default=env, required=not env,
                    help="the reference source tree (default: $PW_REFERENCE_ROOT)")
    args = ap.parse_args()
    copy_fixtures(args.reference)
    torch_expert_goldens(args.reference)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
