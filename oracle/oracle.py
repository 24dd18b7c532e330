"""ctypes/numpy front end for the CPU oracle in pw_oracle.c.

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() and by
bench.py's cpu_baseline / --impl reference legs, as the checker.  The product
path (mimo_prismwing_b200 and its CUDA library) never imports this module.

Each wrapper names the reference function that the C routine restates
(path:line inside the x3haloed/mimo-prismwing tree).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpw_oracle.so")
REF_TOPK_PATH = os.path.join(HERE, "_ref", "libpw_topk_ref.so")

ACC_F32 = 0
ACC_F64 = 1
LAYOUT_PLAIN = 0
LAYOUT_FULL_QKV = 1
LAYOUT_SWA_QKV = 2
EXP_SLEEF = 0
EXP_LIBM = 1

_lib = None


def reference_root() -> str | None:
    """Where the reference source tree is checked out, if anywhere: the
    PW_REFERENCE_ROOT environment variable, else BASELINE.json's
    "reference_path" at the repository root.  None when neither names an
    existing tree (the GPU box has no reference tree)."""
    root = os.environ.get("PW_REFERENCE_ROOT")
    if not root:
        try:
            import json
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                root = json.load(f).get("reference_path")
        except (OSError, ValueError):
            root = None
    return root if root and os.path.isdir(os.path.join(root, "src")) else None


def build() -> None:
    """Compile libpw_oracle.so (and the reference top-k bridge when the reference is present)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    ref = reference_root()
    if ref:
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={ref}"], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = ctypes.CDLL(LIB_PATH)
        _bind(_lib)
    return _lib


def _p(t):
    return ctypes.POINTER(t)


def _bind(L: ctypes.CDLL) -> None:
    u8p, f32p, u32p, u16p = _p(ctypes.c_uint8), _p(ctypes.c_float), _p(ctypes.c_uint32), _p(ctypes.c_uint16)
    sz = ctypes.c_size_t
    L.pwo_decode_e4m3.argtypes = [ctypes.c_uint8]
    L.pwo_decode_e4m3.restype = ctypes.c_float
    L.pwo_round_bf16.argtypes = [ctypes.c_float]
    L.pwo_round_bf16.restype = ctypes.c_float
    L.pwo_encode_e4m3_search.argtypes = [ctypes.c_float, u8p]
    L.pwo_encode_e4m3_rne.argtypes = [ctypes.c_float, u8p]
    L.pwo_dynamic_fp8.argtypes = [f32p, sz, sz, u8p, f32p, f32p]
    L.pwo_validate_fp8.argtypes = [u8p, f32p, sz, sz, f32p, sz, ctypes.c_int, _p(sz)]
    L.pwo_readable_gemv.argtypes = [u8p, f32p, sz, sz, f32p, f32p, ctypes.c_int]
    L.pwo_full_qkv_source_row.argtypes = [sz]
    L.pwo_full_qkv_source_row.restype = sz
    L.pwo_full_qkv_scale_row.argtypes = [sz]
    L.pwo_full_qkv_scale_row.restype = sz
    L.pwo_swa_qkv_source_row.argtypes = [sz]
    L.pwo_swa_qkv_source_row.restype = sz
    L.pwo_blockscaled_linear.argtypes = [u8p, f32p, sz, sz, ctypes.c_int, u8p, f32p, sz, f32p, ctypes.c_int]
    L.pwo_sleef_expf_u10.argtypes = [ctypes.c_float]
    L.pwo_sleef_expf_u10.restype = ctypes.c_float
    L.pwo_sigmoid.argtypes = [ctypes.c_float]
    L.pwo_sigmoid.restype = ctypes.c_float
    L.pwo_staged_swiglu.argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_int]
    L.pwo_staged_swiglu.restype = ctypes.c_float
    L.pwo_router_logits.argtypes = [f32p, sz, u16p, sz, sz, f32p]
    L.pwo_router_logits_f32.argtypes = [f32p, sz, f32p, sz, sz, f32p]
    L.pwo_rms_square_sum.argtypes = [f32p, sz]
    L.pwo_rms_square_sum.restype = ctypes.c_float
    L.pwo_rms_inverse.argtypes = [f32p, sz, ctypes.c_float, f32p]
    L.pwo_rms_norm.argtypes = [f32p, sz, sz, f32p, ctypes.c_float, f32p, f32p]
    L.pwo_residual_add.argtypes = [f32p, f32p, sz, f32p]
    L.pwo_noaux_topk.argtypes = [f32p, f32p, sz, sz, sz, u32p, f32p, f32p, f32p]
    L.pwo_routed_layer.argtypes = [f32p, sz, sz, sz, u32p, f32p, sz, _p(ctypes.c_void_p),
                                   ctypes.c_int, ctypes.c_int, f32p, f32p, f32p]
    L.pwo_schedule.argtypes = [u32p, sz, sz, u32p, u32p]
    L.pwo_round_bf16_array.argtypes = [f32p, f32p, sz]
    L.pwo_decode_e4m3_array.argtypes = [u8p, f32p, sz]
    L.pwo_sleef_expf_array.argtypes = [f32p, f32p, sz]
    L.pwo_sigmoid_array.argtypes = [f32p, f32p, sz]
    L.pwo_staged_swiglu_array.argtypes = [f32p, f32p, f32p, sz, ctypes.c_int]
    L.pwo_set_threads.argtypes = [ctypes.c_int]
    L.pwo_get_threads.restype = ctypes.c_int


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(ctypes.POINTER(t))


def set_threads(n: int) -> None:
    lib().pwo_set_threads(int(n))


def get_threads() -> int:
    return int(lib().pwo_get_threads())


# ---------------------------------------------------------------- scalars
def decode_e4m3(bits: int) -> float:
    """src/lib.rs:7456 decode_f8_e4m3fn."""
    return lib().pwo_decode_e4m3(bits)


def decode_table() -> np.ndarray:
    return np.array([lib().pwo_decode_e4m3(b) for b in range(256)], dtype=np.float32)


def _array_call(fn, v: np.ndarray, *extra) -> np.ndarray:
    v = np.ascontiguousarray(v, dtype=np.float32)
    out = np.empty_like(v)
    fn(_ptr(v, ctypes.c_float), _ptr(out, ctypes.c_float), v.size, *extra)
    return out


def round_bf16(values) -> np.ndarray:
    """src/text_endpoint.rs:2960 round_bf16, elementwise (C routine, exact bits)."""
    return _array_call(lib().pwo_round_bf16_array, values)


def decode_array(codes) -> np.ndarray:
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    out = np.empty(c.shape, np.float32)
    lib().pwo_decode_e4m3_array(_ptr(c, ctypes.c_uint8), _ptr(out, ctypes.c_float), c.size)
    return out


def sleef_expf_array(x) -> np.ndarray:
    return _array_call(lib().pwo_sleef_expf_array, x)


def sigmoid_array(x) -> np.ndarray:
    return _array_call(lib().pwo_sigmoid_array, x)


def round_bf16_bits(values) -> np.ndarray:
    """Vectorised restatement of src/text_endpoint.rs:2960 on raw bits."""
    v = np.ascontiguousarray(values, dtype=np.float32)
    bits = v.view(np.uint32).astype(np.uint64)
    is_special = (bits & 0x7F800000) == 0x7F800000
    is_nan = is_special & ((bits & 0x007FFFFF) != 0)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000) & 0xFFFFFFFF
    nan_bits = ((((bits >> 16) & 0xFFFF) | 0x0040) << 16) & 0xFFFFFFFF
    out = np.where(is_nan, nan_bits, np.where(is_special, bits, rounded)).astype(np.uint32)
    return out.view(np.float32)


def encode_e4m3(value: float, rne: bool = False) -> int:
    """src/text_endpoint.rs:2985 encode_f8_e4m3fn (search), or the exact-RNE form."""
    out = ctypes.c_uint8()
    f = lib().pwo_encode_e4m3_rne if rne else lib().pwo_encode_e4m3_search
    if f(ctypes.c_float(value), ctypes.byref(out)) != 0:
        raise ValueError("E4M3FN encoder requires a finite value in [-448,448]")
    return out.value


def sleef_expf(x: float) -> float:
    return lib().pwo_sleef_expf_u10(x)


def sigmoid(x: float) -> float:
    return lib().pwo_sigmoid(x)


def staged_swiglu(gate: np.ndarray, up: np.ndarray, exp_kind: int = EXP_SLEEF) -> np.ndarray:
    """src/text_endpoint.rs:5336-5342 staged bf16 SwiGLU, elementwise."""
    g = np.ascontiguousarray(gate, dtype=np.float32)
    u = np.ascontiguousarray(up, dtype=np.float32)
    out = np.empty_like(g)
    lib().pwo_staged_swiglu_array(_ptr(g, ctypes.c_float), _ptr(u, ctypes.c_float), _ptr(out, ctypes.c_float),
                                  g.size, exp_kind)
    return out


# ---------------------------------------------------------------- arrays
def dynamic_fp8(x: np.ndarray):
    """src/text_endpoint.rs:3008 dynamic_fp8_activations -> (codes u8, scales f32, dequantized f32)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    codes = np.empty((rows, cols), np.uint8)
    scales = np.empty((rows, cols // 128), np.float32)
    deq = np.empty((rows, cols), np.float32)
    rc = lib().pwo_dynamic_fp8(_ptr(x, ctypes.c_float), rows, cols, _ptr(codes, ctypes.c_uint8),
                              _ptr(scales, ctypes.c_float), _ptr(deq, ctypes.c_float))
    if rc != 0:
        raise ValueError(f"dynamic FP8 activation shape or value mismatch ({rc})")
    return codes, scales, deq


def validate_fp8(weight: np.ndarray, scale: np.ndarray, x: np.ndarray | None, scan: bool = True) -> int:
    """src/lib.rs:1217 validate_fp8_views_internal; 0 or a negative code."""
    weight = np.ascontiguousarray(weight, dtype=np.uint8)
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    at = ctypes.c_size_t(0)
    xp = None
    n = 0
    if x is not None:
        x = np.ascontiguousarray(x, dtype=np.float32)
        xp = _ptr(x, ctypes.c_float)
        n = x.size
    rows, cols = weight.shape
    return lib().pwo_validate_fp8(_ptr(weight, ctypes.c_uint8), _ptr(scale, ctypes.c_float), rows, cols,
                                  xp, n, int(scan), ctypes.byref(at))


def readable_gemv(weight: np.ndarray, scale: np.ndarray, x: np.ndarray, mode: int = ACC_F64) -> np.ndarray:
    """src/lib.rs:1272 mapped_fp8_gemv (x is not quantized); y f32 [rows]."""
    weight = np.ascontiguousarray(weight, dtype=np.uint8)
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = weight.shape
    y = np.empty(rows, np.float32)
    rc = lib().pwo_readable_gemv(_ptr(weight, ctypes.c_uint8), _ptr(scale, ctypes.c_float), rows, cols,
                                 _ptr(x, ctypes.c_float), _ptr(y, ctypes.c_float), mode)
    if rc != 0:
        raise ValueError(f"readable FP8 GEMV failed ({rc})")
    return y


def blockscaled_linear(weight, scale, codes, code_scales, layout: int = LAYOUT_PLAIN,
                       mode: int = ACC_F64) -> np.ndarray:
    """src/wide_metal_moe.rs:404-423 block-scaled equation; returns f32 pre-round [width, rows]."""
    weight = np.ascontiguousarray(weight, dtype=np.uint8)
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    code_scales = np.ascontiguousarray(code_scales, dtype=np.float32)
    rows, cols = weight.shape
    width = codes.shape[0]
    out = np.empty((width, rows), np.float32)
    rc = lib().pwo_blockscaled_linear(_ptr(weight, ctypes.c_uint8), _ptr(scale, ctypes.c_float), rows, cols,
                                      layout, _ptr(codes, ctypes.c_uint8), _ptr(code_scales, ctypes.c_float),
                                      width, _ptr(out, ctypes.c_float), mode)
    if rc != 0:
        raise ValueError(f"block-scaled linear failed ({rc})")
    return out


def full_qkv_source_row(r: int) -> int:
    v = lib().pwo_full_qkv_source_row(r)
    if v == ctypes.c_size_t(-1).value:
        raise ValueError("full-QKV logical row is out of range")
    return v


def full_qkv_scale_row(r: int) -> int:
    v = lib().pwo_full_qkv_scale_row(r)
    if v == ctypes.c_size_t(-1).value:
        raise ValueError("full-QKV logical row is out of range")
    return v


def swa_qkv_source_row(r: int) -> int:
    v = lib().pwo_swa_qkv_source_row(r)
    if v == ctypes.c_size_t(-1).value:
        raise ValueError("SWA-QKV logical row is out of range")
    return v


def router_logits(x: np.ndarray, weight: np.ndarray) -> np.ndarray:
    """Router logits (src/text_endpoint.rs:4350-4358 route_mlp's f32 linear): f32
    fused-multiply-add chains over 256-column slices, added in slice order (the
    pinned order; see pw_oracle.c).  `weight` is the F32 gate.weight (float32)
    or bf16 bits (uint16)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    tokens, hidden = x.shape
    experts = weight.shape[0]
    out = np.empty((tokens, experts), np.float32)
    if weight.dtype == np.float32:
        w = np.ascontiguousarray(weight)
        rc = lib().pwo_router_logits_f32(_ptr(x, ctypes.c_float), tokens, _ptr(w, ctypes.c_float), experts, hidden,
                                         _ptr(out, ctypes.c_float))
    elif weight.dtype in (np.uint16, np.int16):
        w = np.ascontiguousarray(weight).view(np.uint16)
        rc = lib().pwo_router_logits(_ptr(x, ctypes.c_float), tokens, _ptr(w, ctypes.c_uint16), experts, hidden,
                                     _ptr(out, ctypes.c_float))
    else:
        raise TypeError(f"router weight must be float32 or bf16 bits (uint16), not {weight.dtype}")
    if rc != 0:
        raise ValueError("router logits shape mismatch")
    return out


def rms_square_sum(values: np.ndarray) -> np.float32:
    """pytorch_contiguous_inner_square_sum_f32 (src/lib.rs:1905): PyTorch's cascade order."""
    v = np.ascontiguousarray(values, dtype=np.float32).ravel()
    return np.float32(lib().pwo_rms_square_sum(_ptr(v, ctypes.c_float), v.size))


def rms_inverse(values: np.ndarray, epsilon: float) -> np.float32:
    """stable_rms_inverse (src/lib.rs:1890); raises ValueError where the reference returns Err."""
    v = np.ascontiguousarray(values, dtype=np.float32).ravel()
    out = np.zeros(1, np.float32)
    if lib().pwo_rms_inverse(_ptr(v, ctypes.c_float), v.size, ctypes.c_float(epsilon), _ptr(out, ctypes.c_float)):
        raise ValueError("invalid RMSNorm input")
    return out[0]


def rms_norm(x: np.ndarray, weight: np.ndarray, epsilon: float = 1e-5):
    """rms_norm (src/text_endpoint.rs:2939) -> (out f32 [rows, cols], inverse f32 [rows])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    w = np.ascontiguousarray(weight, dtype=np.float32)
    if w.shape != (cols,):
        raise ValueError("RMSNorm shape mismatch")
    out = np.empty_like(x)
    inv = np.empty(rows, np.float32)
    if lib().pwo_rms_norm(_ptr(x, ctypes.c_float), rows, cols, _ptr(w, ctypes.c_float), ctypes.c_float(epsilon),
                          _ptr(out, ctypes.c_float), _ptr(inv, ctypes.c_float)):
        raise ValueError("invalid RMSNorm input")
    return out, inv


def residual_add(residual: np.ndarray, projected: np.ndarray) -> np.ndarray:
    """src/text_endpoint.rs:5576-5580: bf16(residual + projected)."""
    r = np.ascontiguousarray(residual, dtype=np.float32)
    p = np.ascontiguousarray(projected, dtype=np.float32)
    out = np.empty_like(r)
    lib().pwo_residual_add(_ptr(r, ctypes.c_float), _ptr(p, ctypes.c_float), r.size, _ptr(out, ctypes.c_float))
    return out


def noaux_topk(logits: np.ndarray, bias: np.ndarray, top_k: int = 8):
    """src/text_endpoint.rs:4394 pytorch_noaux_routes in canonical order.

    Returns (selected u32 [T,8], weights f32 [T,8], scores f32 [T,E], margin f32 [T], tie_rows)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    bias = np.ascontiguousarray(bias, dtype=np.float32)
    tokens, experts = logits.shape
    sel = np.empty((tokens, top_k), np.uint32)
    wts = np.empty((tokens, top_k), np.float32)
    scores = np.empty((tokens, experts), np.float32)
    margin = np.empty(tokens, np.float32)
    rc = lib().pwo_noaux_topk(_ptr(logits, ctypes.c_float), _ptr(bias, ctypes.c_float), tokens, experts, top_k,
                              _ptr(sel, ctypes.c_uint32), _ptr(wts, ctypes.c_float),
                              _ptr(scores, ctypes.c_float), _ptr(margin, ctypes.c_float))
    if rc < 0:
        raise ValueError(f"noaux top-k failed ({rc})")
    return sel, wts, scores, margin, rc


def schedule(selected: np.ndarray, experts: int):
    sel = np.ascontiguousarray(selected, dtype=np.uint32)
    tokens = sel.shape[0]
    offsets = np.empty(experts + 1, np.uint32)
    order = np.empty(tokens * 8, np.uint32)
    rc = lib().pwo_schedule(_ptr(sel, ctypes.c_uint32), tokens, experts, _ptr(offsets, ctypes.c_uint32),
                            _ptr(order, ctypes.c_uint32))
    if rc != 0:
        raise ValueError("schedule failed")
    return offsets, order


def routed_layer(x: np.ndarray, selected: np.ndarray, weights: np.ndarray, bank: list,
                 mode: int = ACC_F64, exp_kind: int = EXP_SLEEF, want_intermediates: bool = False):
    """src/text_endpoint.rs:5290 routed_mlp_traced with the wide runtime's staging.

    bank[e] = (gate_w, gate_s, up_w, up_s, down_w, down_s) numpy arrays."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    tokens, hidden = x.shape
    intermediate = bank[0][0].shape[0]
    experts = len(bank)
    sel = np.ascontiguousarray(selected, dtype=np.uint32)
    wts = np.ascontiguousarray(weights, dtype=np.float32)
    keep = []
    table = (ctypes.c_void_p * (experts * 6))()
    for e, parts in enumerate(bank):
        for j, a in enumerate(parts):
            a = np.ascontiguousarray(a)
            keep.append(a)
            table[e * 6 + j] = a.ctypes.data
    out = np.empty((tokens, hidden), np.float32)
    hid = np.empty((tokens * 8, intermediate), np.float32) if want_intermediates else None
    down = np.empty((tokens * 8, hidden), np.float32) if want_intermediates else None
    rc = lib().pwo_routed_layer(_ptr(x, ctypes.c_float), tokens, hidden, intermediate,
                                _ptr(sel, ctypes.c_uint32), _ptr(wts, ctypes.c_float), experts,
                                table, mode, exp_kind, _ptr(out, ctypes.c_float),
                                _ptr(hid, ctypes.c_float) if hid is not None else None,
                                _ptr(down, ctypes.c_float) if down is not None else None)
    if rc != 0:
        raise ValueError(f"routed layer failed ({rc})")
    if want_intermediates:
        return out, hid, down
    return out


# ------------------------------------------------------- reference top-k
def reference_topk_unsorted(values: np.ndarray, k: int = 8) -> np.ndarray:
    """Call the reference's own src/pytorch_topk.cpp (compiled into _ref/)."""
    L = ctypes.CDLL(REF_TOPK_PATH)
    L.pw_pytorch_topk_unsorted_f32.argtypes = [_p(ctypes.c_float), ctypes.c_size_t, ctypes.c_size_t,
                                               _p(ctypes.c_uint32)]
    v = np.ascontiguousarray(values, dtype=np.float32)
    out = np.empty(k, np.uint32)
    rc = L.pw_pytorch_topk_unsorted_f32(_ptr(v, ctypes.c_float), v.size, k, _ptr(out, ctypes.c_uint32))
    if rc != 0:
        raise ValueError("reference top-k failed")
    return out
