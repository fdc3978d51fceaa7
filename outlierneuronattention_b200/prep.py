"""Gates + RoPE + cache export in one launch (``hofa_prep_fwd``).

Fuses the layer glue of src/HybridOutlierFactorizedAttention.py
(LotanGutman/OutlierNeuronAttention): ``_compute_gates_optimized`` (:67-95),
``logsigmoid(-gate)`` (:177, :361), in-place RoPE of q/k channels [0, R)
(:180-188, :365-375) and the outlier-cache export / append (:196-198,
:382-384).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _capi
from ._capi import PrepArgs, flat, tview


def prep(q, k, v, gate_w, gate_b, log_gamma, *, mix_w=None, mix_b=None, fixed_mix=None, mix_out=None,
         cos=None, sin=None, R: int = 0, pos0: int = 0, pos0_dev: Optional[torch.Tensor] = None,
         cache_k=None, cache_v=None, use_rope: bool = True) -> None:
    """q, k, v [B,H,N,D] (q/k channels [0,R) rotated in place); gate_w [H,2D],
    gate_b [H]; writes log_gamma [B,H,N] and mix_out [B,H,N]; cache rows
    pos0..pos0+N-1 of cache_k [B,H,L,R] / cache_v [B,H,L,D] when given."""
    vals = flat(tview(q), tview(k), tview(v), tview(gate_w), tview(gate_b), tview(mix_w), tview(mix_b),
                tview(fixed_mix), tview(cos), tview(sin), tview(log_gamma), tview(mix_out),
                tview(cache_k), tview(cache_v), int(R), int(pos0),
                0 if pos0_dev is None else pos0_dev.data_ptr(), 1 if use_rope else 0)
    _capi.call("hofa_prep_fwd", PrepArgs, vals, _capi.stream_handle(q.device))
