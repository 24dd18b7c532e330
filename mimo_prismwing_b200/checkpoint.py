"""Checkpoint ingestion over the C ABI: safetensors shards and PWEXPRT1 expert
containers, mapped read-only and validated fail-closed by the library
(csrc/pw_checkpoint.cpp), then uploaded into HBM expert banks.

Names follow the reference: `MappedSafetensors.open` / `tensor` /
`tensor_count` (src/lib.rs:784-976), `repack_expert_container` and
`verify_expert_container` (src/lib.rs:7190-7347).  Opening and reading files
needs no GPU; uploads go to the runtime's device.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import _lib

PW_OK = 0

_NP_DTYPES = {"U8": np.uint8, "I8": np.int8, "F8_E4M3": np.uint8, "F8_E4M3FN": np.uint8, "F8_E5M2": np.uint8,
              "BOOL": np.bool_, "U16": np.uint16, "I16": np.int16, "F16": np.float16, "BF16": np.uint16,
              "U32": np.uint32, "I32": np.int32, "F32": np.float32, "U64": np.uint64, "I64": np.int64,
              "F64": np.float64}


class TensorView(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("dtype", ctypes.c_char_p), ("rank", ctypes.c_uint32),
                ("shape", ctypes.c_uint64 * 8), ("data", ctypes.c_void_p), ("bytes", ctypes.c_uint64)]


class CheckpointError(RuntimeError):
    """A non-zero status from the checkpoint entry points (the reference's Err(String))."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def _bind(L) -> None:
    if getattr(L, "_pw_checkpoint_bound", False):
        return
    vp, u32, sz, cp = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_size_t, ctypes.c_char_p
    L.pw_safetensors_open.argtypes = [cp, ctypes.POINTER(vp), cp, sz]
    L.pw_container_open.argtypes = [cp, ctypes.POINTER(vp), cp, sz]
    L.pw_container_repack.argtypes = [cp, cp, ctypes.POINTER(cp), u32, cp, sz]
    L.pw_tensor_file_close.argtypes = [vp]
    L.pw_tensor_file_close.restype = None
    L.pw_tensor_file_count.argtypes = [vp, ctypes.POINTER(u32)]
    L.pw_tensor_file_at.argtypes = [vp, u32, ctypes.POINTER(TensorView)]
    L.pw_tensor_file_find.argtypes = [vp, cp, ctypes.POINTER(TensorView)]
    L.pw_tensor_upload.argtypes = [vp, ctypes.POINTER(vp), u32, cp, cp, ctypes.POINTER(ctypes.c_uint64), u32,
                                   ctypes.POINTER(vp), cp, sz]
    L.pw_device_free.argtypes = [vp, vp]
    L.pw_bank_load.argtypes = [vp, ctypes.POINTER(vp), u32, u32, u32, u32, ctypes.POINTER(vp), cp, sz]
    L._pw_checkpoint_bound = True


def _lib_bound():
    L = _lib.load()
    _bind(L)
    return L


@dataclass
class Tensor:
    """MappedTensorView: metadata plus the bytes in the read-only mapping."""
    name: str
    dtype: str
    shape: tuple
    data: int
    nbytes: int

    def numpy(self) -> np.ndarray:
        """A copy of the tensor as numpy (e4m3 and bf16 as their raw bits)."""
        buf = (ctypes.c_uint8 * self.nbytes).from_address(self.data)
        return np.frombuffer(bytes(buf), dtype=_NP_DTYPES[self.dtype]).reshape(self.shape)


class TensorFile:
    """An opened safetensors shard or PWEXPRT1 container (pw_tensor_file)."""

    def __init__(self, handle: ctypes.c_void_p, path: str):
        self._h = handle
        self.path = path

    @classmethod
    def _open(cls, fn, path: str) -> "TensorFile":
        L = _lib_bound()
        h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        st = getattr(L, fn)(path.encode(), ctypes.byref(h), err, 512)
        if st != PW_OK:
            raise CheckpointError(st, err.value.decode(errors="replace"))
        return cls(h, path)

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib_bound().pw_tensor_file_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @staticmethod
    def _view(v: TensorView) -> Tensor:
        return Tensor(v.name.decode(), v.dtype.decode(), tuple(v.shape[i] for i in range(v.rank)), v.data or 0,
                      v.bytes)

    def tensor_count(self) -> int:
        n = ctypes.c_uint32()
        _lib_bound().pw_tensor_file_count(self._h, ctypes.byref(n))
        return n.value

    def names(self) -> list:
        L = _lib_bound()
        out = []
        for i in range(self.tensor_count()):
            v = TensorView()
            L.pw_tensor_file_at(self._h, i, ctypes.byref(v))
            out.append(v.name.decode())
        return out

    def tensor(self, name: str) -> Tensor:
        v = TensorView()
        st = _lib_bound().pw_tensor_file_find(self._h, name.encode(), ctypes.byref(v))
        if st != PW_OK:
            raise CheckpointError(st, f"tensor is absent: {name}")
        return self._view(v)


class MappedSafetensors(TensorFile):
    """src/lib.rs:784 MappedSafetensors::open."""

    @classmethod
    def open(cls, path: str) -> "MappedSafetensors":
        return cls._open("pw_safetensors_open", path)


class ExpertContainer(TensorFile):
    """A verified PWEXPRT1 container (src/lib.rs:7282 verify_expert_container)."""

    @classmethod
    def open(cls, path: str) -> "ExpertContainer":
        return cls._open("pw_container_open", path)


def verify_expert_container(path: str) -> ExpertContainer:
    return ExpertContainer.open(path)


def repack_expert_container(source: str, output: str, tensor_names: Sequence[str]) -> ExpertContainer:
    """src/lib.rs:7190: copy the named tensors into a new container, then verify it."""
    L = _lib_bound()
    names = (ctypes.c_char_p * max(1, len(tensor_names)))(*[n.encode() for n in tensor_names])
    err = ctypes.create_string_buffer(512)
    st = L.pw_container_repack(source.encode(), output.encode(), names, len(tensor_names), err, 512)
    if st != PW_OK:
        raise CheckpointError(st, err.value.decode(errors="replace"))
    return ExpertContainer.open(output)


def _handles(files: Sequence[TensorFile]):
    return (ctypes.c_void_p * len(files))(*[f._h for f in files])


class DeviceBuffer:
    """A device allocation made by pw_tensor_upload; torch.as_tensor(buf,
    device="cuda") views it through __cuda_array_interface__."""

    _TYPESTR = {"F32": "<f4", "BF16": "<u2", "F8_E4M3": "|u1", "U8": "|u1", "I32": "<i4", "F16": "<f2"}

    def __init__(self, rt, ptr: int, dtype: str, shape: tuple):
        self._rt, self.ptr, self.dtype, self.shape = rt, ptr, dtype, shape

    @property
    def __cuda_array_interface__(self):
        return {"shape": self.shape, "typestr": self._TYPESTR[self.dtype], "data": (self.ptr, False), "version": 3}

    def free(self) -> None:
        if self.ptr:
            _lib_bound().pw_device_free(self._rt._rt, ctypes.c_void_p(self.ptr))
            self.ptr = 0


def upload(rt, files: Sequence[TensorFile], name: str, dtype: Optional[str] = None,
           shape: Optional[Sequence[int]] = None) -> DeviceBuffer:
    """pw_tensor_upload: one tensor (found in exactly one file) into a new device buffer."""
    L = _lib_bound()
    ptr = ctypes.c_void_p()
    err = ctypes.create_string_buffer(512)
    shp = (ctypes.c_uint64 * len(shape))(*shape) if shape is not None else None
    st = L.pw_tensor_upload(rt._rt, _handles(files), len(files), name.encode(), dtype.encode() if dtype else None,
                            shp, len(shape) if shape is not None else 0, ctypes.byref(ptr), err, 512)
    if st != PW_OK:
        raise CheckpointError(st, err.value.decode(errors="replace"))
    t = None
    for f in files:
        try:
            t = f.tensor(name)
            break
        except CheckpointError:
            continue
    return DeviceBuffer(rt, ptr.value, t.dtype, t.shape)


def load_bank(rt, files: Sequence[TensorFile], layer: int, first_expert: int, n_experts: int):
    """pw_bank_load: routed experts [first, first + n) of `layer` into a bank
    (the bank owns the device memory; the runtime destroys it on close)."""
    L = _lib_bound()
    bank = ctypes.c_void_p()
    err = ctypes.create_string_buffer(512)
    st = L.pw_bank_load(rt._rt, _handles(files), len(files), layer, first_expert, n_experts, ctypes.byref(bank),
                        err, 512)
    if st != PW_OK:
        raise CheckpointError(st, err.value.decode(errors="replace"))
    rt._banks.append(bank)
    return bank
