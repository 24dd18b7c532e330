"""Python mirror of the reference's routed-MoE runtime over the C ABI.

The class and method names follow the reference's Rust runtime
(`WideMetalMoeRuntime`, src/wide_metal_moe.rs:165-1316) so that tests read
like the reference's own: `compile`, `compile_with_fused_gate_up`,
`execute_fp8_linear`, `execute`, `execute_fused_gate_up`.  Every call goes
through include/pw_cuda.h into mimo_prismwing_b200/lib/libpw_cuda.so; there is
no CPU fallback, and loading fails loudly when the library is missing.

Tensors: weights and scales are torch CUDA tensors (uint8 e4m3 bytes, float32
scale grids); activations may be CUDA tensors (device I/O) or CPU tensors /
numpy arrays (host I/O: the call copies in and out, as the reference's
commit + wait_until_completed does).
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np
import torch

from . import _lib

PW_OK = 0
LAYOUT_PLAIN = 0
LAYOUT_FULL_QKV = 1
LAYOUT_SWA_QKV = 2
OUTPUT_F32 = 0x100
MEM_DEVICE = 0
MEM_HOST = 1
MEM_ASYNC = 2
EP_NCCL_TRANSPORT = 1
RUNTIME_FUSED_GATE_UP = 1
ROUTER_F32 = 0
ROUTER_BF16 = 1
NORM_F32 = 0
NORM_BF16 = 1

ERRORS = {
    -1: "argument", -2: "shape", -3: "nonfinite", -4: "device_flags", -5: "cuda", -6: "nccl",
    -7: "timeout", -8: "schedule", -9: "unsupported",
}


class PrismwingError(RuntimeError):
    """A non-zero status from the C ABI (the reference's Err(String))."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[{ERRORS.get(status, status)}] {message}")
        self.status = status
        self.kind = ERRORS.get(status, str(status))


class Fp8Tensor(ctypes.Structure):
    _fields_ = [("weight", ctypes.c_void_p), ("scale", ctypes.c_void_p), ("rows", ctypes.c_uint32),
                ("cols", ctypes.c_uint32), ("scale_rows", ctypes.c_uint32), ("scale_cols", ctypes.c_uint32)]


class ExpertWeights(ctypes.Structure):
    _fields_ = [("gate", Fp8Tensor), ("up", Fp8Tensor), ("down", Fp8Tensor)]


class ExpertBinding(ctypes.Structure):
    _fields_ = [("expert", ctypes.c_uint32), ("count", ctypes.c_uint32), ("positions", ctypes.c_void_p),
                ("route_weights", ctypes.c_void_p), ("weights", ExpertWeights)]


class Router(ctypes.Structure):
    _fields_ = [("weight", ctypes.c_void_p), ("bias", ctypes.c_void_p), ("experts", ctypes.c_uint32),
                ("hidden", ctypes.c_uint32), ("top_k", ctypes.c_uint32), ("weight_dtype", ctypes.c_uint32)]


class Norm(ctypes.Structure):
    _fields_ = [("weight", ctypes.c_void_p), ("hidden", ctypes.c_uint32), ("weight_dtype", ctypes.c_uint32),
                ("epsilon", ctypes.c_float)]


class Stats(ctypes.Structure):
    _fields_ = [("wall_ms", ctypes.c_double), ("device_ms", ctypes.c_float), ("error_flags", ctypes.c_uint32),
                ("unique_experts", ctypes.c_uint32), ("expert_rows", ctypes.c_uint32),
                ("boundary_tie_rows", ctypes.c_uint32), ("weight_bytes", ctypes.c_uint64)]

    def as_dict(self) -> dict:
        return {k: getattr(self, k) for k, _ in self._fields_}


class Profile(ctypes.Structure):
    _fields_ = [("quantize_ms", ctypes.c_float), ("router_ms", ctypes.c_float), ("schedule_ms", ctypes.c_float),
                ("gate_up_ms", ctypes.c_float), ("down_ms", ctypes.c_float), ("combine_ms", ctypes.c_float),
                ("projection_ms", ctypes.c_float), ("launches", ctypes.c_uint32)]

    def as_dict(self) -> dict:
        return {k: getattr(self, k) for k, _ in self._fields_}


# ------------------------------------------------------------------ bindings
@dataclass
class WideProjectionBinding:
    """One e4m3 matrix + f32 scale grid on the GPU (src/wide_metal_moe.rs:80)."""
    weight: torch.Tensor  # uint8 [rows, cols], CUDA
    scale: torch.Tensor   # float32 [scale_rows, scale_cols], CUDA

    @property
    def rows(self) -> int:
        return int(self.weight.shape[0])

    @property
    def columns(self) -> int:
        return int(self.weight.shape[1])

    def c(self) -> Fp8Tensor:
        w, s = self.weight, self.scale
        if not (w.is_cuda and s.is_cuda and w.dtype == torch.uint8 and s.dtype == torch.float32):
            raise PrismwingError(-1, "projection weight must be CUDA uint8 and scale CUDA float32")
        if not (w.is_contiguous() and s.is_contiguous()):
            raise PrismwingError(-1, "projection tensors must be contiguous")
        return Fp8Tensor(w.data_ptr(), s.data_ptr(), w.shape[0], w.shape[1], s.shape[0], s.shape[1])


@dataclass
class WideExpertBinding:
    """An expert's placements and projections (src/wide_metal_moe.rs:88)."""
    expert: int
    positions: Sequence[int]
    route_weights: Sequence[float]
    gate: WideProjectionBinding
    up: WideProjectionBinding
    down: WideProjectionBinding

    def weights_c(self) -> ExpertWeights:
        return ExpertWeights(self.gate.c(), self.up.c(), self.down.c())


@dataclass
class Execution:
    """WideLinearExecution / WideMoeExecution (src/wide_metal_moe.rs:97-111)."""
    output: torch.Tensor
    wall_ms: float
    device_ms: float
    unique_experts: int = 0
    expert_rows: int = 0
    boundary_tie_rows: int = 0
    weight_bytes: int = 0
    selected: Optional[torch.Tensor] = None
    weights: Optional[torch.Tensor] = None


def _as_f32(x) -> torch.Tensor:
    if isinstance(x, np.ndarray):
        x = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    if x.dtype != torch.float32:
        x = x.float()
    return x.contiguous()


class WideMoeRuntime:
    """B200 counterpart of the reference's WideMetalMoeRuntime."""

    def __init__(self, device: int = 0, fused_gate_up: bool = True):
        self._L = _lib.load()
        rt = ctypes.c_void_p()
        st = self._L.pw_runtime_create(device, RUNTIME_FUSED_GATE_UP if fused_gate_up else 0, ctypes.byref(rt))
        if st != PW_OK:
            raise PrismwingError(st, f"pw_runtime_create failed on device {device}")
        self._rt = rt
        self.device = device
        self.fused_gate_up = fused_gate_up
        self._banks = []
        self._bank_refs = []

    # reference constructors (src/wide_metal_moe.rs:165-171)
    @classmethod
    def compile(cls, device: int = 0) -> "WideMoeRuntime":
        return cls(device, fused_gate_up=False)

    @classmethod
    def compile_with_fused_gate_up(cls, device: int = 0) -> "WideMoeRuntime":
        return cls(device, fused_gate_up=True)

    def close(self) -> None:
        for b in self._banks:
            self._L.pw_bank_destroy(b)
        self._banks = []
        self._bank_refs = []
        if getattr(self, "_rt", None):
            self._L.pw_runtime_destroy(self._rt)
            self._rt = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------ plumbing
    def _check(self, status: int) -> None:
        if status != PW_OK:
            raise PrismwingError(status, self._L.pw_last_error(self._rt).decode())

    def last_error(self) -> str:
        return self._L.pw_last_error(self._rt).decode()

    def set_stream(self, stream: Optional[torch.cuda.Stream]) -> None:
        self._check(self._L.pw_set_stream(self._rt, ctypes.c_void_p(stream.cuda_stream if stream else 0)))

    def synchronize(self) -> None:
        self._check(self._L.pw_synchronize(self._rt))

    def set_profiling(self, enable: bool) -> None:
        """Per-kernel CUDA-event timing of subsequent synchronous calls."""
        self._check(self._L.pw_set_profiling(self._rt, 1 if enable else 0))

    def last_profile(self) -> dict:
        p = Profile()
        self._check(self._L.pw_last_profile(self._rt, ctypes.byref(p)))
        return p.as_dict()

    def error_flags(self) -> int:
        f = ctypes.c_uint32()
        self._check(self._L.pw_read_error_flags(self._rt, ctypes.byref(f)))
        return f.value

    def _io(self, x, out_shape, out_dtype=torch.float32):
        x = _as_f32(x)
        mem = MEM_DEVICE if x.is_cuda else MEM_HOST
        dev = x.device if x.is_cuda else torch.device("cpu")
        out = torch.empty(out_shape, dtype=out_dtype, device=dev)
        return x, out, mem

    # -------------------------------------------------------- primitives
    def quantize(self, x):
        """dynamic_fp8_activations (src/text_endpoint.rs:3008) -> (codes u8, scales f32)."""
        x = _as_f32(x)
        rows, cols = x.shape
        mem = MEM_DEVICE if x.is_cuda else MEM_HOST
        codes = torch.empty((rows, cols), dtype=torch.uint8, device=x.device)
        scales = torch.empty((rows, cols // 128 if cols % 128 == 0 else 1), dtype=torch.float32, device=x.device)
        self._check(self._L.pw_quantize_fp8(self._rt, ctypes.c_void_p(x.data_ptr()), rows, cols,
                                            ctypes.c_void_p(codes.data_ptr()), ctypes.c_void_p(scales.data_ptr()),
                                            mem))
        return codes, scales

    def validate(self, binding: WideProjectionBinding) -> None:
        """validate_fp8_views_internal (src/lib.rs:1217); raises on a bad byte or scale."""
        t = binding.c()
        bad = ctypes.c_uint64()
        self._check(self._L.pw_validate_fp8(self._rt, ctypes.byref(t), ctypes.byref(bad)))

    def _io_async(self, x, out_shape, asynchronous, out):
        """(x, out, mem, stats pointer) for a call that may be enqueued without
        waiting (PW_MEM_ASYNC: device I/O, no stats; CUDA-graph capturable once
        the same call has run before)."""
        if asynchronous:
            if not x.is_cuda:
                raise PrismwingError(-1, "asynchronous calls need device I/O")
            if out is None:
                out = torch.empty(out_shape, dtype=torch.float32, device=x.device)
            return x, out, MEM_DEVICE | MEM_ASYNC, None
        x, o, mem = self._io(x, out_shape)
        return x, (out if out is not None and x.is_cuda else o), mem, Stats()

    def fp8_gemv(self, x, binding: WideProjectionBinding, asynchronous: bool = False,
                 out: Optional[torch.Tensor] = None) -> Execution:
        """Readable projection (src/lib.rs:1272 mapped_fp8_gemv): x f32 [w, cols] -> f32 [w, rows]."""
        x = _as_f32(x)
        if x.dim() == 1:
            x = x.unsqueeze(0)
        x, out, mem, st = self._io_async(x, (x.shape[0], binding.rows), asynchronous, out)
        t = binding.c()
        self._check(self._L.pw_fp8_gemv(self._rt, ctypes.byref(t), ctypes.c_void_p(x.data_ptr()), x.shape[0],
                                        ctypes.c_void_p(out.data_ptr()), mem, ctypes.byref(st) if st else None))
        return Execution(out, st.wall_ms if st else 0.0, st.device_ms if st else 0.0,
                         weight_bytes=st.weight_bytes if st else 0)

    def execute_fp8_linear(self, x, binding: WideProjectionBinding, full_qkv_layout: bool = False,
                           layout: Optional[int] = None, f32_output: bool = False, asynchronous: bool = False,
                           out: Optional[torch.Tensor] = None) -> Execution:
        """src/wide_metal_moe.rs:241: quantize, block-scaled projection, bf16 round.

        Like the reference, a [14848, 4096] projection selects the SWA-QKV row map
        and full_qkv_layout=True the full-QKV map.  f32_output skips the final
        bf16 round (PW_OUTPUT_F32)."""
        x = _as_f32(x)
        if layout is None:
            if full_qkv_layout:
                layout = LAYOUT_FULL_QKV
            elif binding.rows == 14848 and binding.columns == 4096:
                layout = LAYOUT_SWA_QKV
            else:
                layout = LAYOUT_PLAIN
        if f32_output:
            layout |= OUTPUT_F32
        x, out, mem, st = self._io_async(x, (x.shape[0], binding.rows), asynchronous, out)
        t = binding.c()
        self._check(self._L.pw_fp8_linear(self._rt, ctypes.byref(t), layout, ctypes.c_void_p(x.data_ptr()),
                                          x.shape[0], ctypes.c_void_p(out.data_ptr()), mem,
                                          ctypes.byref(st) if st else None))
        return Execution(out, st.wall_ms if st else 0.0, st.device_ms if st else 0.0,
                         weight_bytes=st.weight_bytes if st else 0)

    def expert_forward(self, x, gate: WideProjectionBinding, up: WideProjectionBinding,
                       down: WideProjectionBinding, asynchronous: bool = False,
                       out: Optional[torch.Tensor] = None) -> Execution:
        """One routed expert at weight 1 (src/text_endpoint.rs:5311-5346)."""
        x = _as_f32(x)
        x, out, mem, st = self._io_async(x, (x.shape[0], down.rows), asynchronous, out)
        w = ExpertWeights(gate.c(), up.c(), down.c())
        self._check(self._L.pw_expert_forward(self._rt, ctypes.byref(w), ctypes.c_void_p(x.data_ptr()), x.shape[0],
                                              ctypes.c_void_p(out.data_ptr()), mem,
                                              ctypes.byref(st) if st else None))
        return Execution(out, st.wall_ms if st else 0.0, st.device_ms if st else 0.0,
                         weight_bytes=st.weight_bytes if st else 0)

    def dense_mlp(self, x, gate: WideProjectionBinding, up: WideProjectionBinding,
                  down: WideProjectionBinding) -> Execution:
        """dense_mlp (src/text_endpoint.rs:4266): layer 0's dense FP8 MLP
        (gate/up [16384, 4096], down [4096, 16384] for MiMo-V2.5)."""
        x = _as_f32(x)
        x, out, mem = self._io(x, (x.shape[0], down.rows))
        w = ExpertWeights(gate.c(), up.c(), down.c())
        st = Stats()
        self._check(self._L.pw_dense_mlp(self._rt, ctypes.byref(w), ctypes.c_void_p(x.data_ptr()), x.shape[0],
                                         ctypes.c_void_p(out.data_ptr()), mem, ctypes.byref(st)))
        return Execution(out, st.wall_ms, st.device_ms, weight_bytes=st.weight_bytes)

    def route(self, x, router_weight: torch.Tensor, bias: torch.Tensor):
        """route_mlp + pytorch_noaux_routes (src/text_endpoint.rs:4342-4470).

        router_weight: CUDA [E, H], float32 (the checkpoint's F32 gate.weight) or
        bf16 (or int16 bits); bias CUDA f32 [E].
        Returns (selected int64 [T, 8], weights f32 [T, 8], stats dict)."""
        x = _as_f32(x)
        r = self._router(router_weight, bias)
        mem = MEM_DEVICE if x.is_cuda else MEM_HOST
        sel = torch.empty((x.shape[0], 8), dtype=torch.int32, device=x.device)
        wts = torch.empty((x.shape[0], 8), dtype=torch.float32, device=x.device)
        st = Stats()
        self._check(self._L.pw_route(self._rt, ctypes.byref(r), ctypes.c_void_p(x.data_ptr()), x.shape[0],
                                     ctypes.c_void_p(sel.data_ptr()), ctypes.c_void_p(wts.data_ptr()), mem,
                                     ctypes.byref(st)))
        return sel.long() & 0xFFFFFFFF, wts, st.as_dict()

    @staticmethod
    def _router(w: torch.Tensor, bias: torch.Tensor) -> Router:
        """pw_router for a CUDA float32 (PW_ROUTER_F32) or bf16/int16 (PW_ROUTER_BF16) weight."""
        if w.dtype == torch.float32:
            dtype = ROUTER_F32
        elif w.dtype in (torch.bfloat16, torch.int16):
            dtype = ROUTER_BF16
        else:
            raise PrismwingError(-1, f"router weight must be float32 or bf16, not {w.dtype}")
        if not (w.is_cuda and bias.is_cuda and bias.dtype == torch.float32):
            raise PrismwingError(-1, "router weight and bias must be CUDA tensors, bias float32")
        if not (w.is_contiguous() and bias.is_contiguous()):
            raise PrismwingError(-1, "router tensors must be contiguous")
        return Router(w.data_ptr(), bias.data_ptr(), w.shape[0], w.shape[1], 8, dtype)

    @staticmethod
    def _norm(weight: torch.Tensor, epsilon: float) -> Norm:
        """pw_norm for a CUDA float32 (PW_NORM_F32) or bf16/int16 (PW_NORM_BF16) weight."""
        if weight.dtype == torch.float32:
            dtype = NORM_F32
        elif weight.dtype in (torch.bfloat16, torch.int16):
            dtype = NORM_BF16
        else:
            raise PrismwingError(-1, f"norm weight must be float32 or bf16, not {weight.dtype}")
        if not (weight.is_cuda and weight.is_contiguous() and weight.dim() == 1):
            raise PrismwingError(-1, "norm weight must be a contiguous 1-D CUDA tensor")
        return Norm(weight.data_ptr(), weight.shape[0], dtype, float(epsilon))

    def rms_norm(self, x, weight: torch.Tensor, epsilon: float = 1e-5):
        """rms_norm (src/text_endpoint.rs:2939): (y f32 [rows, H], inverse f32 [rows])."""
        x = _as_f32(x)
        n = self._norm(weight, epsilon)
        x, out, mem = self._io(x, tuple(x.shape))
        inv = torch.empty((x.shape[0],), dtype=torch.float32, device=out.device)
        self._check(self._L.pw_rms_norm(self._rt, ctypes.byref(n), ctypes.c_void_p(x.data_ptr()), x.shape[0],
                                        ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(inv.data_ptr()), mem, None))
        return out, inv

    # ------------------------------------------------------------ layers
    def execute(self, x, experts: Sequence[WideExpertBinding]) -> Execution:
        """src/wide_metal_moe.rs:836 execute: host-built schedule, whole layer on device."""
        return self._execute(x, experts)

    def execute_fused_gate_up(self, x, experts: Sequence[WideExpertBinding]) -> Execution:
        """src/wide_metal_moe.rs:844 execute_fused_gate_up (this runtime must be fused)."""
        if not self.fused_gate_up:
            raise PrismwingError(-1, "fused gate/up pipelines were not requested")
        return self._execute(x, experts)

    def _execute(self, x, experts: Sequence[WideExpertBinding]) -> Execution:
        x = _as_f32(x)
        rows = x.shape[0]
        x, out, mem = self._io(x, (rows, x.shape[1]))
        arr = (ExpertBinding * len(experts))()
        keep = []
        for i, e in enumerate(experts):
            pos = np.ascontiguousarray(np.asarray(e.positions, dtype=np.uint32))
            wts = np.ascontiguousarray(np.asarray(e.route_weights, dtype=np.float32))
            keep += [pos, wts]
            arr[i] = ExpertBinding(e.expert, len(pos), pos.ctypes.data, wts.ctypes.data, e.weights_c())
        st = Stats()
        self._check(self._L.pw_moe_execute(self._rt, ctypes.c_void_p(x.data_ptr()), rows, arr, len(experts),
                                           ctypes.c_void_p(out.data_ptr()), mem, ctypes.byref(st)))
        return Execution(out, st.wall_ms, st.device_ms, st.unique_experts, st.expert_rows, weight_bytes=st.weight_bytes)

    def create_bank(self, experts: Sequence[tuple]) -> ctypes.c_void_p:
        """Register experts [(gate, up, down) WideProjectionBinding triples]; validates every byte."""
        arr = (ExpertWeights * len(experts))()
        for i, (g, u, d) in enumerate(experts):
            arr[i] = ExpertWeights(g.c(), u.c(), d.c())
        bank = ctypes.c_void_p()
        self._check(self._L.pw_bank_create(self._rt, arr, len(experts), ctypes.byref(bank)))
        self._banks.append(bank)
        # the library keeps raw device pointers: hold the tensors as long as the bank
        self._bank_refs.append(list(experts))
        return bank

    # ------------------------------------------------- expert parallelism
    @staticmethod
    def ep_unique_id() -> bytes:
        """A fresh NCCL communicator id (128 bytes) for pw_ep_init; create it on
        one rank and send it to the others."""
        L = _lib.load()
        buf = ctypes.create_string_buffer(128)
        rc = L.pw_ep_unique_id(buf, 128)
        if rc != 0:
            raise PrismwingError(rc, "pw_ep_unique_id failed (is libnccl.so.2 loadable?)")
        return buf.raw

    def ep_init(self, rank: int, world: int, uid: bytes, timeout_ms: int = 60000, max_tokens: int = 2048,
                hidden: int = 0, local_experts: int = 0, nccl_transport: bool = False) -> None:
        """Join the expert-parallel group (collective).  max_tokens bounds the
        tokens per rank and layer (same on every rank); with hidden and
        local_experts the peer-memory windows are mapped here; nccl_transport
        moves the rows with NCCL send/recv instead of peer-memory stores."""
        buf = ctypes.create_string_buffer(bytes(uid), len(uid))
        self._check(self._L.pw_ep_init(self._rt, rank, world, buf, len(uid), timeout_ms, max_tokens, hidden,
                                       local_experts, EP_NCCL_TRANSPORT if nccl_transport else 0))

    def ep_moe_layer(self, x, router_weight: torch.Tensor, bias: torch.Tensor, bank,
                     want_routes: bool = False, stats: bool = True, asynchronous: bool = False,
                     out: Optional[torch.Tensor] = None) -> Execution:
        """Collective routed layer over this rank's tokens; `bank` holds this
        rank's experts (rank g: experts [g n, (g + 1) n))."""
        x = _as_f32(x)
        T, H = x.shape
        r = self._router(router_weight, bias)
        mem = MEM_DEVICE if x.is_cuda else MEM_HOST
        if asynchronous:
            if not x.is_cuda:
                raise PrismwingError(-1, "asynchronous calls need device I/O")
            mem |= MEM_ASYNC
            stats = False
        if out is None:
            out = torch.empty((T, H), dtype=torch.float32, device=x.device)
        sel = torch.empty((T, 8), dtype=torch.int32, device=x.device) if want_routes else None
        wts = torch.empty((T, 8), dtype=torch.float32, device=x.device) if want_routes else None
        st = Stats()
        self._check(self._L.pw_ep_moe_layer(
            self._rt, ctypes.byref(r), bank, ctypes.c_void_p(x.data_ptr() if T else 0), T,
            ctypes.c_void_p(out.data_ptr() if T else 0),
            ctypes.c_void_p(sel.data_ptr() if sel is not None and T else 0),
            ctypes.c_void_p(wts.data_ptr() if wts is not None and T else 0), mem,
            ctypes.byref(st) if stats else None))
        return Execution(out, st.wall_ms, st.device_ms, st.unique_experts, st.expert_rows, st.boundary_tie_rows,
                         st.weight_bytes, sel, wts)

    def moe_layer(self, x, router_weight: torch.Tensor, bias: torch.Tensor, bank,
                  want_routes: bool = False, stats: bool = True, asynchronous: bool = False,
                  out: Optional[torch.Tensor] = None) -> Execution:
        """routed_mlp_metal_wide_configured (src/text_endpoint.rs:4750) fully on the device."""
        x = _as_f32(x)
        T, H = x.shape
        r = self._router(router_weight, bias)
        mem = MEM_DEVICE if x.is_cuda else MEM_HOST
        if asynchronous:
            if not x.is_cuda:
                raise PrismwingError(-1, "asynchronous calls need device I/O")
            mem |= MEM_ASYNC
            stats = False
        if out is None:
            out = torch.empty((T, H), dtype=torch.float32, device=x.device)
        sel = torch.empty((T, 8), dtype=torch.int32, device=x.device) if want_routes else None
        wts = torch.empty((T, 8), dtype=torch.float32, device=x.device) if want_routes else None
        st = Stats()
        self._check(self._L.pw_moe_layer(
            self._rt, ctypes.byref(r), bank, ctypes.c_void_p(x.data_ptr()), T, ctypes.c_void_p(out.data_ptr()),
            ctypes.c_void_p(sel.data_ptr() if sel is not None else 0),
            ctypes.c_void_p(wts.data_ptr() if wts is not None else 0), mem,
            ctypes.byref(st) if stats else None))
        return Execution(out, st.wall_ms, st.device_ms, st.unique_experts, st.expert_rows, st.boundary_tie_rows,
                         st.weight_bytes, sel, wts)

    def moe_block(self, residual, norm_weight: torch.Tensor, epsilon: float, router_weight: torch.Tensor,
                  bias: torch.Tensor, bank, want_routes: bool = False, stats: bool = True,
                  asynchronous: bool = False, out: Optional[torch.Tensor] = None, expert_parallel: bool = False
                  ) -> Execution:
        """The MoE half of a decoder layer (src/text_endpoint.rs:5507-5580):
        out = bf16(residual + routed_layer(rms_norm(residual))).  With
        expert_parallel the call is pw_ep_moe_block (collective)."""
        x = _as_f32(residual)
        T, H = x.shape
        n = self._norm(norm_weight, epsilon)
        r = self._router(router_weight, bias)
        mem = MEM_DEVICE if x.is_cuda else MEM_HOST
        if asynchronous:
            if not x.is_cuda:
                raise PrismwingError(-1, "asynchronous calls need device I/O")
            mem |= MEM_ASYNC
            stats = False
        if out is None:
            out = torch.empty((T, H), dtype=torch.float32, device=x.device)
        sel = torch.empty((T, 8), dtype=torch.int32, device=x.device) if want_routes else None
        wts = torch.empty((T, 8), dtype=torch.float32, device=x.device) if want_routes else None
        st = Stats()
        fn = self._L.pw_ep_moe_block if expert_parallel else self._L.pw_moe_block
        self._check(fn(self._rt, ctypes.byref(n), ctypes.byref(r), bank, ctypes.c_void_p(x.data_ptr() if T else 0), T,
                       ctypes.c_void_p(out.data_ptr() if T else 0),
                       ctypes.c_void_p(sel.data_ptr() if sel is not None and T else 0),
                       ctypes.c_void_p(wts.data_ptr() if wts is not None and T else 0), mem,
                       ctypes.byref(st) if stats else None))
        return Execution(out, st.wall_ms, st.device_ms, st.unique_experts, st.expert_rows, st.boundary_tie_rows,
                         st.weight_bytes, sel, wts)
