"""Shared helpers for the GPU parity tests: host copies for the oracle and the
parity metrics (tolerances quoted from the north-star: dequantization and
route indices bit-exact, projections and layers within relative 2e-3 of the
f64-accumulated oracle, measured norm-wise and as max|d|/max|ref|)."""
import numpy as np
import torch

REL_TOL = 2e-3


def host(t):
    return t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)


def rel_errors(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    d = got - ref
    l2 = np.linalg.norm(d) / max(np.linalg.norm(ref), 1e-30)
    mx = np.max(np.abs(d)) / max(np.max(np.abs(ref)), 1e-30)
    return l2, mx


def assert_close(got, ref, tol=REL_TOL, what=""):
    l2, mx = rel_errors(got, ref)
    assert l2 <= tol and mx <= tol, f"{what}: rel L2 {l2:.3e}, max rel {mx:.3e} (tol {tol})"


def bf16_ulp(v):
    """Spacing of bf16 values at |v| (2^(e-7) for normal v)."""
    a = np.maximum(np.abs(np.asarray(v, dtype=np.float64)), 2.0 ** -126)
    return 2.0 ** (np.floor(np.log2(a)) - 7)


def assert_close_bf16(got, ref, tol=REL_TOL, what="", max_ulps=2, max_frac=5e-3):
    """Parity for outputs with bf16 staging points (expert and layer outputs).

    The f64 oracle and the GPU round at the same bf16 boundaries, but their f32
    pre-round values differ by reassociation; where a value sits next to a bf16
    midpoint the two round to adjacent bf16 numbers (the effect the reference
    itself measured between its Metal and CPU paths).  So: relative L2 <= tol,
    every element within tol * max|ref| except flips of at most `max_ulps`
    bf16 ulps, and such flips on at most `max_frac` of the elements."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    l2, mx = rel_errors(got, ref)
    assert l2 <= tol, f"{what}: rel L2 {l2:.3e} (tol {tol})"
    d = np.abs(got - ref)
    big = d > tol * np.max(np.abs(ref))
    ulps = d / bf16_ulp(np.maximum(np.abs(ref), np.abs(got)))
    assert np.all(ulps[big] <= max_ulps + 1e-9), f"{what}: {np.max(ulps[big]):.2f} bf16 ulps beyond tolerance"
    assert np.mean(big) <= max_frac, f"{what}: {np.mean(big):.2%} of elements beyond {tol} of max"


def bank_arrays(bank):
    """[(gate_w, gate_s, up_w, up_s, down_w, down_s) numpy] for the oracle."""
    out = []
    for g, u, d in bank:
        out.append((host(g.weight), host(g.scale), host(u.weight), host(u.scale), host(d.weight), host(d.scale)))
    return out
