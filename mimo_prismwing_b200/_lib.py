"""Loader for the in-tree CUDA library (mimo_prismwing_b200/lib/libpw_cuda.so).

There is no fallback: if the library is missing or does not export every
symbol of include/pw_cuda.h, loading raises.  torch is imported first so that
its CUDA runtime and NCCL are the ones resolved in this process.
"""
from __future__ import annotations

import ctypes
import os
import re

import torch  # noqa: F401  (load order: torch's CUDA libraries first)

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB_PATH = os.path.join(PKG, "lib", "libpw_cuda.so")
HEADER = os.path.join(ROOT, "include", "pw_cuda.h")

_lib = None


def header_symbols(path: str = HEADER) -> list[str]:
    """Function names declared in a C header of this repository."""
    with open(path) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pw_[a-z0-9_]+)\s*\(", text)))


def _p(t):
    return ctypes.POINTER(t)


def _bind(L: ctypes.CDLL) -> None:
    vp, u32, i32 = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int
    L.pw_abi_version.restype = i32
    L.pw_runtime_create.argtypes = [i32, u32, _p(vp)]
    L.pw_runtime_destroy.argtypes = [vp]
    L.pw_runtime_destroy.restype = None
    L.pw_last_error.argtypes = [vp]
    L.pw_last_error.restype = ctypes.c_char_p
    L.pw_set_stream.argtypes = [vp, vp]
    L.pw_synchronize.argtypes = [vp]
    L.pw_read_error_flags.argtypes = [vp, _p(u32)]
    L.pw_quantize_fp8.argtypes = [vp, vp, u32, u32, vp, vp, u32]
    L.pw_validate_fp8.argtypes = [vp, vp, _p(ctypes.c_uint64)]
    L.pw_fp8_gemv.argtypes = [vp, vp, vp, u32, vp, u32, vp]
    L.pw_fp8_linear.argtypes = [vp, vp, u32, vp, u32, vp, u32, vp]
    L.pw_expert_forward.argtypes = [vp, vp, vp, u32, vp, u32, vp]
    L.pw_route.argtypes = [vp, vp, vp, u32, vp, vp, u32, vp]
    L.pw_moe_execute.argtypes = [vp, vp, u32, vp, u32, vp, u32, vp]
    L.pw_bank_create.argtypes = [vp, vp, u32, _p(vp)]
    L.pw_bank_destroy.argtypes = [vp]
    L.pw_bank_destroy.restype = None
    L.pw_moe_layer.argtypes = [vp, vp, vp, vp, u32, vp, vp, vp, u32, vp]
    L.pw_ep_unique_id.argtypes = [vp, u32]
    L.pw_ep_init.argtypes = [vp, i32, i32, vp, u32, u32, u32, u32, u32, u32]
    L.pw_ep_rank.argtypes = [vp, _p(i32), _p(i32)]
    L.pw_ep_plan.argtypes = [vp, u32, u32, u32, vp, vp, vp, vp, vp]
    L.pw_ep_moe_layer.argtypes = [vp, vp, vp, vp, u32, vp, vp, vp, u32, vp]
    L.pw_rms_norm.argtypes = [vp, vp, vp, u32, vp, vp, u32, vp]
    L.pw_dense_mlp.argtypes = [vp, vp, vp, u32, vp, u32, vp]
    L.pw_moe_block.argtypes = [vp, vp, vp, vp, vp, u32, vp, vp, vp, u32, vp]
    L.pw_ep_moe_block.argtypes = [vp, vp, vp, vp, vp, u32, vp, vp, vp, u32, vp]
    L.pw_set_profiling.argtypes = [vp, i32]
    L.pw_last_profile.argtypes = [vp, vp]
    for name in header_symbols():
        getattr(L, name)  # raises AttributeError if an entry point is missing


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m mimo_prismwing_b200.build` "
                "(there is no CPU fallback for the CUDA path)")
        L = ctypes.CDLL(LIB_PATH)
        _bind(L)
        _lib = L
    return _lib
