"""Prefill outlier-attention operator with the reference's name and signature.

``exact_attention_triton`` keeps the reference's name
(src/exact_attention.py:163-188 of LotanGutman/OutlierNeuronAttention) so
callers can swap the import; it runs ``hofa_prefill_outlier_fwd`` of
libhofa_b200.so (hand-written sm_100a CUDA, no Triton).  Semantics:
``out += mix_g * softmax(sm_scale * q_r k_r^T, causal) v`` over the first
``r`` channels of q/k; ``out`` defaults to zeros like ``v``.
"""
from __future__ import annotations

import torch

from . import _capi
from ._capi import OutlierArgs, flat, tview


def exact_attention_triton(q, k, v, r, sm_scale, mix_g, out=None, split_k=None, *, q_offset: int = 0,
                           accumulate: bool = True):
    """q, k: [B,H,T,>=r] (RoPE-rotated in [:r]); v: [B,H,T,D]; mix_g [B,H,T].
    ``split_k`` is accepted for signature compatibility and ignored (as in the
    reference).  Keyword-only extensions: ``q_offset`` (key j is visible to
    query i iff j <= i + q_offset; q may then be a suffix block of the
    sequence) and ``accumulate`` (False overwrites ``out``)."""
    if out is None:
        out = torch.zeros(q.shape[0], q.shape[1], q.shape[2], v.shape[-1], dtype=v.dtype, device=v.device)
    vals = flat(tview(q), tview(k), tview(v), tview(mix_g), tview(out), int(r), int(q_offset),
                float(sm_scale), 1 if accumulate else 0)
    _capi.call("hofa_prefill_outlier_fwd", OutlierArgs, vals, _capi.stream_handle(q.device))
    return out
