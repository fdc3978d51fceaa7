"""Prefill GLA operator with the reference's name and signature.

``chunk_gla_inlier_fwd`` mirrors src/chunk_gla_inlier.py:153-237 of
LotanGutman/OutlierNeuronAttention: it returns ``(Y, states_out)`` where
``Y`` is ``(1 - mix_g) * gla_scale * RMSNorm(y_I)`` when both ``mix_g`` and
``gla_scale`` are given (otherwise the raw GLA output ``y_I``) and
``states_out`` is the final float32 state in the reference's padded buffer
``[B, H, max(16, 2^ceil(log2 j)), max(16, 2^ceil(log2 D))]`` (callers slice
``[:, :, :j, :D]``).  It runs ``hofa_prefill_gla_fwd`` of libhofa_b200.so.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _capi
from ._capi import GlaArgs, flat, tview

_WS = {}


def _pow2_at_least16(n: int) -> int:
    return max(1 << max(0, (n - 1)).bit_length(), 16)


def _workspace(device, B, H, T, D, R, nseg) -> torch.Tensor:
    """The call's workspace, cached per (device, stream): the tensor-core GLA
    keeps its chunk tickets and publication flags there, so two calls that
    may run at the same time (on different streams) must not share one."""
    nbytes = int(_capi.lib().hofa_gla_workspace_size(B, H, T, D, R, 64, nseg))
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, torch.cuda.current_stream(idx).cuda_stream)
    ws = _WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WS[key] = ws
    return ws


def gla_forward(Q, K, V, log_gamma, r, *, log_alpha=None, mix_g=None, gla_scale=None, y=None,
                state_out=None, initial_state=None, eps: float = 1e-5, chunk_size: int = 64,
                num_segments: int = 0):
    """Low-level launch: writes ``y`` ([B,H,T,D], allocated if None) and the
    final state into ``state_out`` ([B,H,D-r,D] float32, optional).
    ``initial_state`` seeds the recurrence (zero when None)."""
    B, H, T, D = Q.shape
    if y is None:
        y = torch.empty(B, H, T, D, dtype=Q.dtype, device=Q.device)
    ws = _workspace(Q.device, B, H, T, D, r, num_segments)
    vals = flat(tview(Q), tview(K), tview(V), tview(log_gamma), tview(log_alpha), tview(mix_g),
                tview(gla_scale), tview(initial_state), tview(y), tview(state_out),
                int(r), int(chunk_size), float(eps), int(num_segments), ws.data_ptr(), ws.numel())
    _capi.call("hofa_prefill_gla_fwd", GlaArgs, vals, _capi.stream_handle(Q.device))
    return y


def chunk_gla_inlier_fwd(Q, K, V, log_gamma, r, chunk_size, log_alpha=None, mix_g=None, gla_scale=None,
                         out=None, states_in=None, requires_grad=False, *, eps: float = 1e-5,
                         initial_state: Optional[torch.Tensor] = None):
    """Chunked GLA over channels [r:D] of Q/K (drop-in for the reference op).

    Q, K, V: [B,H,T,D]; log_gamma [B,H,T]; r outlier channels skipped;
    chunk_size is a tiling hint (the result does not depend on it beyond
    rounding).  ``log_alpha`` ([1,H,1,D-r]) enables per-channel decay;
    ``mix_g`` ([B,H,T] or [B,H,T,1]) with ``gla_scale`` ([1,H,1,D] or [H,D])
    enables the fused ``(1-mix)*gla_scale*RMSNorm`` epilogue (eps 1e-5 as in
    the reference).  ``out`` receives Y when given.  ``states_in`` and
    ``requires_grad`` belong to the reference's training path (per-chunk state
    dump for backward), which this inference library does not build.
    Keyword-only extension: ``initial_state`` ([B,H,D-r,D] float32) seeds the
    recurrence (sequence-sharded prefill).
    """
    if requires_grad or states_in is not None:
        raise NotImplementedError("the per-chunk state dump for backward (requires_grad) is training-only "
                                  "and not part of this inference library")
    B, H, T, D = Q.shape
    j = D - r
    states_out = torch.zeros(B, H, _pow2_at_least16(j), _pow2_at_least16(D), dtype=torch.float32, device=Q.device)
    fuse = mix_g is not None and gla_scale is not None
    y = gla_forward(Q, K, V, log_gamma, r, log_alpha=log_alpha, mix_g=mix_g if fuse else None,
                    gla_scale=gla_scale if fuse else None, y=out, state_out=states_out[:, :, :j, :D],
                    initial_state=initial_state, eps=eps, chunk_size=chunk_size)
    return y, states_out
