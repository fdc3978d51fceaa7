"""Decode operator with the reference's name and signature.

``fused_hofa_decode`` mirrors src/hofa_decode_triton.py:342-476 of
LotanGutman/OutlierNeuronAttention (same positional/keyword arguments,
same return value: a new ``Y`` of shape [B,H,1,D] in q's dtype, with
``state_I_out`` written in place) and runs the single fused sm_100a kernel
behind ``hofa_decode_fwd`` in libhofa_b200.so.
"""
from __future__ import annotations

import threading
from typing import Dict, Optional, Tuple

import torch

from . import _capi
from ._capi import DecodeArgs, flat, tview

FP32_EPS = float(torch.finfo(torch.float32).eps)

_WS: Dict[Tuple[int, int, int, int], torch.Tensor] = {}
_WS_LOCK = threading.Lock()


def decode_workspace(device: torch.device, B: int, H: int, D: int) -> torch.Tensor:
    """Zero-filled decode workspace for (device, B, H, D), sized for the
    largest split count.  Allocated once per shape (outside any CUDA-graph
    capture, on first use); every launch leaves it reusable.  Replaces the
    reference's ``_get_cached_split_workspace`` (hofa_decode_triton.py:20-27)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, B, H, D)
    ws = _WS.get(key)
    if ws is None:
        with _WS_LOCK:
            ws = _WS.get(key)
            if ws is None:
                nbytes = _capi.lib().hofa_decode_workspace_size(B, H, D, 0)
                ws = torch.zeros(nbytes, dtype=torch.uint8, device=torch.device("cuda", idx))
                _WS[key] = ws
    return ws


def choose_split(B: int, H: int, seq_len: int, device: Optional[torch.device] = None) -> int:
    """Split count the library picks for this shape (see hofa_decode_choose_split)."""
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    return int(_capi.lib().hofa_decode_choose_split(B, H, seq_len, sms))


def decode_args(q, k, v, cache_k, cache_v, state_I_in, state_I_out, log_gamma, mix_g, norm_w,
                R, seq_len, sm_scale, y, split_k=None, log_alpha=None, eps=FP32_EPS,
                seq_len_dev: Optional[torch.Tensor] = None, workspace: Optional[torch.Tensor] = None):
    """The packed ``hofa_decode_args`` value tuple (for callers that launch
    the same step repeatedly, e.g. under CUDA-graph capture)."""
    B, H, _, D = q.shape
    ws = workspace if workspace is not None else decode_workspace(q.device, B, H, D)
    return flat(tview(q), tview(k), tview(v), tview(cache_k if R > 0 else None),
                tview(cache_v if R > 0 else None), tview(state_I_in), tview(state_I_out),
                tview(log_gamma), tview(mix_g), tview(norm_w), tview(log_alpha), tview(y),
                int(R), int(seq_len), 0 if seq_len_dev is None else seq_len_dev.data_ptr(),
                float(sm_scale), float(eps), int(split_k or 0), ws.data_ptr(), ws.numel())


def fused_hofa_decode(q, k, v, cache_k, cache_v, state_I_in, state_I_out, log_gamma, mix_g, norm_w,
                      R, seq_len, sm_scale, split_k=None, log_alpha=None, *, eps: float = FP32_EPS,
                      seq_len_dev: Optional[torch.Tensor] = None):
    """One HOFA decode step of the attention core (drop-in for the reference op).

    q, k, v: [B,H,1,D] (q[..., :R] RoPE-rotated); cache_k [B,H,L,R];
    cache_v [B,H,L,D]; state_I_in/out [B,H,D-R,D] float32 (state_I_out is
    written); log_gamma, mix_g [B,H,1]; norm_w [H,D]; R outlier channels;
    seq_len cache rows to attend; sm_scale logit scale.  ``split_k`` overrides
    the automatic cache split.  ``log_alpha`` ([1,H,1,D-R]) enables the
    per-channel decay exponent.  Keyword-only extensions: ``eps`` (RMSNorm;
    the reference uses float32 eps) and ``seq_len_dev`` (an int32 CUDA scalar
    read at run time instead of ``seq_len``, for CUDA-graph replay).
    Returns Y [B,H,1,D] in q's dtype.
    """
    B, H, N, D = q.shape
    assert N == 1, "fused_hofa_decode expects a single token (N=1)"
    y = torch.empty_like(q)
    vals = decode_args(q, k, v, cache_k, cache_v, state_I_in, state_I_out, log_gamma, mix_g, norm_w,
                       R, seq_len, sm_scale, y, split_k, log_alpha, eps, seq_len_dev)
    _capi.call("hofa_decode_fwd", DecodeArgs, vals, _capi.stream_handle(q.device))
    return y


def read_status(device: torch.device, B: int, H: int, D: int) -> int:
    """Status word of the decode workspace (1 = a device seq_len was clamped)."""
    ws = decode_workspace(device, B, H, D)
    out = _capi.ctypes.c_int32(0)
    st = _capi.lib().hofa_decode_read_status(ws.data_ptr(), _capi.stream_handle(device), _capi.ctypes.byref(out))
    if st != 0:
        raise _capi.HofaError("hofa_decode_read_status", st, _capi.lib().hofa_last_error().decode())
    return int(out.value)


def fused_hofa_decode_step(q, k, v, cache_k, cache_v, state_I_in, state_I_out, norm_w, R, seq_len, sm_scale,
                           gate_w, gate_b, *, mix_w=None, mix_b=None, fixed_mix=None, cos=None, sin=None,
                           log_alpha=None, eps: float = FP32_EPS, seq_len_dev: Optional[torch.Tensor] = None,
                           split_k=None, log_gamma_out: Optional[torch.Tensor] = None,
                           mix_out: Optional[torch.Tensor] = None):
    """One decode step of the layer with the new token's prep fused in
    (``hofa_decode_step_fwd``): the gates on the un-rotated q, k
    (src/HybridOutlierFactorizedAttention.py:67-95, :361), RoPE of channels
    [0, R) at position ``seq_len - 1`` (:365-375), the cache append at that row
    (:382-384) and ``fused_hofa_decode`` over rows [0, seq_len) (:386-416).

    q, k, v: [B,H,1,D] un-rotated projections of the new token; cache_k
    [B,H,L,R] and cache_v [B,H,L,D] pre-allocated (row ``seq_len - 1`` is
    written); state_I_in/out [B,H,D-R,D] float32; gate_w [H,2D], gate_b [H];
    the blend from ``mix_w``/``mix_b`` or ``fixed_mix``; RoPE tables ``cos``,
    ``sin`` (no RoPE when None).  ``seq_len_dev`` (int32 CUDA scalar) replaces
    ``seq_len`` for CUDA-graph replay.  q and k are left unspecified.
    Returns (Y [B,H,1,D], log_gamma [B,H,1] float32, mix [B,H,1])."""
    B, H, N, D = q.shape
    assert N == 1, "a decode step takes one token (N=1)"
    y = torch.empty_like(q)
    lg = log_gamma_out if log_gamma_out is not None else torch.empty(B, H, 1, dtype=torch.float32, device=q.device)
    mx = mix_out if mix_out is not None else torch.empty(B, H, 1, dtype=q.dtype, device=q.device)
    dvals = decode_args(q, k, v, cache_k, cache_v, state_I_in, state_I_out, lg, mx, norm_w, R, seq_len, sm_scale, y,
                        split_k, log_alpha, eps, seq_len_dev)
    pvals = flat(tview(q), tview(k), tview(v), tview(gate_w), tview(gate_b), tview(mix_w), tview(mix_b),
                 tview(fixed_mix), tview(cos), tview(sin), tview(lg), tview(mx), tview(cache_k), tview(cache_v),
                 int(R), 0, 0, 1 if cos is not None else 0)
    L = _capi.lib()
    dbuf = _capi.FORMATS[DecodeArgs].pack(*dvals)
    pbuf = _capi.FORMATS[_capi.PrepArgs].pack(*pvals)
    status = L.hofa_decode_step_fwd(dbuf, pbuf, _capi.stream_handle(q.device))
    if status != _capi.HOFA_OK:
        raise _capi.HofaError("hofa_decode_step_fwd", status, L.hofa_last_error().decode())
    return y, lg, mx
