"""ctypes binding of libhofa_b200.so (the C ABI declared in include/hofa.h).

The structures below mirror include/hofa.h field for field.  A call packs its
argument structure with one ``struct.pack`` (format derived from the ctypes
layout, so the byte offsets are the C compiler's) and passes the buffer's
address; the return status is turned into an exception carrying
``hofa_last_error()``.  There is no CPU path: tensors must live on a CUDA
device and the library must be built (``python -m outlierneuronattention_b200.build``).
"""
from __future__ import annotations

import ctypes
import os
import struct
import threading
from ctypes import c_float, c_int32, c_int64, c_size_t, c_void_p
from typing import Optional

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libhofa_b200.so")

HOFA_OK = 0
STATUS_NAMES = {1: "HOFA_ERR_INVALID_ARGUMENT", 2: "HOFA_ERR_UNSUPPORTED", 3: "HOFA_ERR_MISALIGNED",
                4: "HOFA_ERR_WORKSPACE", 5: "HOFA_ERR_CUDA"}
DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


class HofaError(RuntimeError):
    """A non-zero hofa_status from the library."""

    def __init__(self, fn: str, status: int, message: str):
        super().__init__(f"{fn} failed with {STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class HofaTensor(ctypes.Structure):
    _fields_ = [("data", c_void_p), ("dtype", c_int32), ("ndim", c_int32),
                ("shape", c_int64 * 4), ("stride", c_int64 * 4)]


def _T(*names):
    return [(n, HofaTensor) for n in names]


class DecodeArgs(ctypes.Structure):
    _fields_ = _T("q", "k", "v", "cache_k", "cache_v", "state_in", "state_out", "log_gamma", "mix_g",
                  "norm_w", "log_alpha", "y") + [
        ("R", c_int32), ("seq_len", c_int32), ("seq_len_dev", c_void_p), ("sm_scale", c_float),
        ("eps", c_float), ("split_k", c_int32), ("workspace", c_void_p), ("workspace_bytes", c_size_t)]


class GlaArgs(ctypes.Structure):
    _fields_ = _T("q", "k", "v", "log_gamma", "log_alpha", "mix_g", "gla_scale", "state_init", "y",
                  "state_out") + [
        ("R", c_int32), ("chunk_size", c_int32), ("eps", c_float), ("num_segments", c_int32),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t)]


class OutlierArgs(ctypes.Structure):
    _fields_ = _T("q", "k", "v", "mix_g", "out") + [
        ("R", c_int32), ("q_offset", c_int32), ("sm_scale", c_float), ("accumulate", c_int32)]


class PrepArgs(ctypes.Structure):
    _fields_ = _T("q", "k", "v", "gate_w", "gate_b", "mix_w", "mix_b", "fixed_mix", "cos", "sin",
                  "log_gamma", "mix_out", "cache_k", "cache_v") + [
        ("R", c_int32), ("pos0", c_int32), ("pos0_dev", c_void_p), ("use_rope", c_int32)]


class LinearArgs(ctypes.Structure):
    _fields_ = _T("x", "weight", "norm_w", "residual", "y") + [("input_mode", c_int32), ("eps", c_float)]


def _pack_format(cls) -> str:
    """struct format reproducing the C layout of ``cls`` (offsets from ctypes)."""
    fmt, pos = "<", 0
    for name, ctype in cls._fields_:
        off = getattr(cls, name).offset
        if off > pos:
            fmt += f"{off - pos}x"
            pos = off
        if ctype is HofaTensor:
            fmt += "Qii4q4q"
            pos += ctypes.sizeof(HofaTensor)
        elif ctype in (c_int32,):
            fmt += "i"; pos += 4
        elif ctype is c_float:
            fmt += "f"; pos += 4
        elif ctype in (c_void_p, c_size_t):
            fmt += "Q"; pos += 8
        else:
            raise TypeError(ctype)
    tail = ctypes.sizeof(cls) - pos
    if tail:
        fmt += f"{tail}x"
    assert struct.calcsize(fmt) == ctypes.sizeof(cls)
    return fmt


FORMATS = {cls: struct.Struct(_pack_format(cls)) for cls in (DecodeArgs, GlaArgs, OutlierArgs, PrepArgs, LinearArgs)}

ABSENT = (0, 0, 0, 1, 1, 1, 1, 0, 0, 0, 0)


_PAD_SHAPE = ((1, 1, 1, 1), (1, 1, 1), (1, 1), (1,), ())
_PAD_STRIDE = ((0, 0, 0, 0), (0, 0, 0), (0, 0), (0,), ())


def tview(t: Optional[torch.Tensor]):
    """The hofa_tensor fields of a CUDA tensor (or of an absent optional one)."""
    if t is None:
        return ABSENT
    code = DTYPE_CODES.get(t.dtype)
    if code is None:
        raise TypeError(f"unsupported dtype {t.dtype} (float32, bfloat16, float16)")
    if not t.is_cuda:
        raise ValueError("HOFA kernels take CUDA tensors only (this library has no CPU path)")
    nd = t.dim()
    if nd == 4:
        return (t.data_ptr(), code, 4, *t.shape, *t.stride())
    if nd > 4:
        raise ValueError(f"tensors of at most 4 dims, got {nd}")
    return (t.data_ptr(), code, nd, *t.shape, *_PAD_SHAPE[nd], *t.stride(), *_PAD_STRIDE[nd])


_lib = None
_lib_lock = threading.Lock()


def lib():
    """Load libhofa_b200.so once; raise if it is missing (no fallback)."""
    global _lib
    if _lib is None:
        with _lib_lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(f"{LIB_PATH} is missing: build it with "
                                      "`python -m outlierneuronattention_b200.build`")
                L = ctypes.CDLL(LIB_PATH)
                for fn in ("hofa_decode_fwd", "hofa_prefill_gla_fwd", "hofa_prefill_outlier_fwd", "hofa_prep_fwd",
                           "hofa_lm_linear_fwd"):
                    getattr(L, fn).restype = ctypes.c_int
                    getattr(L, fn).argtypes = [c_void_p, c_void_p]
                L.hofa_decode_step_fwd.restype = ctypes.c_int
                L.hofa_decode_step_fwd.argtypes = [c_void_p, c_void_p, c_void_p]
                L.hofa_last_error.restype = ctypes.c_char_p
                L.hofa_abi_version.restype = c_int32
                L.hofa_decode_workspace_size.restype = c_size_t
                L.hofa_decode_workspace_size.argtypes = [c_int32] * 4
                L.hofa_decode_choose_split.restype = c_int32
                L.hofa_decode_choose_split.argtypes = [c_int32] * 4
                L.hofa_decode_read_status.restype = ctypes.c_int
                L.hofa_decode_read_status.argtypes = [c_void_p, c_void_p, ctypes.POINTER(c_int32)]
                L.hofa_prefill_read_status.restype = ctypes.c_int
                L.hofa_prefill_read_status.argtypes = [c_void_p, ctypes.POINTER(c_int32)]
                L.hofa_gla_workspace_size.restype = c_size_t
                L.hofa_gla_workspace_size.argtypes = [c_int32] * 7
                if L.hofa_abi_version() != 1:
                    raise ImportError("libhofa_b200.so ABI version mismatch")
                _lib = L
    return _lib


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def call(fn_name: str, cls, values: tuple, stream: int) -> None:
    """Pack ``values`` as a ``cls`` structure and call ``fn_name`` on ``stream``."""
    L = lib()
    buf = FORMATS[cls].pack(*values)
    status = getattr(L, fn_name)(buf, stream)
    if status != HOFA_OK:
        raise HofaError(fn_name, status, L.hofa_last_error().decode())


def flat(*items):
    """Flatten tensor views (tuples) and scalars into one value tuple."""
    out = []
    for it in items:
        if type(it) is tuple:
            out += it
        else:
            out.append(it)
    return tuple(out)
