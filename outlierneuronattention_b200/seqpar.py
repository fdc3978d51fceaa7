"""Sequence-sharded prefill of the HOFA attention core (long contexts over N GPUs).

A long prompt (e.g. B=1, T=65536 tokens) is cut into 2N equal blocks
and rank r owns blocks r and 2N-1-r ("zig-zag"), so that every rank gets the
same amount of causal attention work.  One exchange step per layer, one
process per GPU over ``torch.distributed`` (NCCL on GPUs):

* outlier attention: every rank needs the rotated outlier keys K_O and the
  values V of all earlier tokens.  They are all-gathered (issued
  asynchronously before the GLA passes, so the transfer overlaps them) and
  placed at their sequence positions; each local block then attends to the
  key prefix ending at its own last token (``q_offset`` = the block's first
  absolute position);
* GLA: each local block first runs from a zero state, giving its end state
  S_b and its total log decay G_b.  These ([B,H,J,D] fp32 + [B,H] or
  [B,H,J]) are all-gathered, every rank forms the start state of each block
  by the prefix recurrence ``S_in[i+1] = exp(G_i) * S_in[i] + S_i`` over the
  2N blocks (the reference's carried-state recurrence,
  src/chunk_gla_inlier.py:86-126, applied per block instead of per chunk),
  and the block is run again from its start state with the fused
  ``(1-mix) * gla_scale * RMSNorm`` epilogue (RMSNorm is not linear, so the
  normalised output has to wait for the start state);
* the attention output is then added into the GLA output (as in the layer).

The compute functions default to this library's CUDA operators
(``gla_forward`` and ``exact_attention_triton``); they are parameters so that
the exchange logic can be checked on CPU ranks against another implementation
of the same operators.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from .chunk_gla_inlier import gla_forward
from .exact_attention import exact_attention_triton
from .hofa_decode import FP32_EPS

Block = Tuple[int, int]


def zigzag_blocks(T: int, world: int, rank: int) -> List[Block]:
    """[start, end) token ranges owned by ``rank`` when T tokens are cut into
    2*world equal blocks: blocks ``rank`` and ``2*world - 1 - rank``."""
    nb = 2 * world
    if T % nb != 0:
        raise ValueError(f"sequence length {T} must be a multiple of 2 * world = {nb}")
    bl = T // nb
    return [(rank * bl, (rank + 1) * bl), ((nb - 1 - rank) * bl, (nb - rank) * bl)]


def block_owner(i: int, world: int) -> Tuple[int, int]:
    """(rank, local block index) of global block ``i`` under zig-zag sharding."""
    return (i, 0) if i < world else (2 * world - 1 - i, 1)


def _group_info(group) -> Tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def _all_gather(t: torch.Tensor, world: int, group, async_op: bool = False):
    parts = [torch.empty_like(t) for _ in range(world)]
    if world == 1:
        parts[0].copy_(t)
        return parts, None
    work = dist.all_gather(parts, t.contiguous(), group=group, async_op=async_op)
    return parts, work


def sharded_attention_core(Q, K, V, log_gamma, mix, r: int, sm_scale: float, gla_scale, T: int, *,
                           group=None, log_alpha=None, eps: float = FP32_EPS,
                           gla: Callable = gla_forward, attn: Callable = exact_attention_triton):
    """The attention core of one rank of a sequence-sharded prefill.

    Q, K, V: [B,H,Tl,D] this rank's tokens (its two zig-zag blocks, in order,
    concatenated along T; Tl = T / world), with RoPE already applied to the
    first r channels of Q and K at the tokens' absolute positions;
    log_gamma [B,H,Tl] float32 and mix [B,H,Tl] (as produced by the layer's
    gate step); gla_scale [1,H,1,D]; T the whole sequence length.
    Returns (Y [B,H,Tl,D] for this rank's tokens, S_end [B,H,D-r,D] float32:
    the GLA state after all T tokens, identical on every rank).
    """
    world, rank = _group_info(group)
    B, H, Tl, D = Q.shape
    J = D - r
    blocks = zigzag_blocks(T, world, rank)
    bl = T // (2 * world)
    if Tl != 2 * bl:
        raise ValueError(f"rank holds {Tl} tokens, expected 2 blocks of {bl}")
    local = [slice(0, bl), slice(bl, 2 * bl)]

    # 1. start the K_O / V exchange (overlaps the first GLA pass)
    kv = torch.cat([K[..., :r], V], dim=-1).contiguous()        # [B,H,Tl,r+D]
    kv_parts, kv_work = _all_gather(kv, world, group, async_op=True)

    # 2. GLA from a zero state per local block: end state and total decay
    S_loc = torch.empty(2, B, H, J, D, dtype=torch.float32, device=Q.device)
    scratch = torch.empty(B, H, bl, D, dtype=Q.dtype, device=Q.device)
    dec_shape = (2, B, H, J) if log_alpha is not None else (2, B, H)
    G_loc = torch.empty(dec_shape, dtype=torch.float32, device=Q.device)
    for i, sl in enumerate(local):
        gla(Q[:, :, sl], K[:, :, sl], V[:, :, sl], log_gamma[:, :, sl], r, log_alpha=log_alpha,
            y=scratch, state_out=S_loc[i], eps=eps)
        g = log_gamma[:, :, sl].float().sum(-1)                 # [B,H]
        if log_alpha is not None:
            g = g[..., None] * torch.exp(log_alpha.float().reshape(1, H, J))
        G_loc[i] = g

    # 3. exchange block states, prefix recurrence over the 2*world blocks
    S_parts, _ = _all_gather(S_loc, world, group)
    G_parts, _ = _all_gather(G_loc, world, group)
    S = torch.zeros(B, H, J, D, dtype=torch.float32, device=Q.device)
    S_in = []
    for i in range(2 * world):
        S_in.append(S)
        owner, li = block_owner(i, world)
        dec = torch.exp(G_parts[owner][li])
        dec = dec[..., None, None] if log_alpha is None else dec[..., None]
        S = dec * S + S_parts[owner][li]
    S_end = S

    # 4. GLA again from each local block's start state, fused epilogue
    Y = torch.empty(B, H, Tl, D, dtype=Q.dtype, device=Q.device)
    for i, ((a, _), sl) in enumerate(zip(blocks, local)):
        gi = a // bl
        gla(Q[:, :, sl], K[:, :, sl], V[:, :, sl], log_gamma[:, :, sl], r, log_alpha=log_alpha,
            mix_g=mix[:, :, sl], gla_scale=gla_scale, y=Y[:, :, sl], initial_state=S_in[gi].contiguous(),
            eps=eps)

    # 5. outlier attention of each local block against its key prefix
    if kv_work is not None:
        kv_work.wait()
    KV = torch.empty(B, H, T, r + D, dtype=Q.dtype, device=Q.device)
    for s in range(world):
        for j, (a, e) in enumerate(zigzag_blocks(T, world, s)):
            KV[:, :, a:e] = kv_parts[s][:, :, j * bl:(j + 1) * bl]
    for (a, e), sl in zip(blocks, local):
        attn(Q[:, :, sl], KV[:, :, :e, :r], KV[:, :, :e, r:], r, sm_scale, mix[:, :, sl], out=Y[:, :, sl],
             q_offset=a)
    return Y, S_end


def sharded_layer_forward(layer, x_local: torch.Tensor, T: int, group=None, return_state: bool = False):
    """Prefill of a ``HybridOutlierFactorizedAttention`` layer with the
    sequence sharded over the ranks of ``group``.

    x_local: [B, T/world, d_model], this rank's tokens (its two zig-zag blocks
    concatenated); T the whole sequence length.  Returns this rank's rows of
    the layer output ([B, T/world, d_model]), and with ``return_state`` also
    the GLA state after all T tokens (every rank holds it).  Hybrid layers
    only (0 < r < d_head, no width split)."""
    if not (0 < layer.r < layer.d_head) or layer.forced_mha_heads > 0:
        raise NotImplementedError("sequence-sharded prefill covers hybrid layers (0 < r < d_head, no width split)")
    world, rank = _group_info(group)
    B, Tl, _ = x_local.shape
    dtype_in = x_local.dtype
    Q, K, V = layer._project(x_local)
    bl = T // (2 * world)
    lg = torch.empty(B, layer.num_heads, Tl, dtype=torch.float32, device=Q.device)
    mix = torch.empty(B, layer.num_heads, Tl, dtype=Q.dtype, device=Q.device)
    for i, (a, _) in enumerate(zigzag_blocks(T, world, rank)):
        sl = slice(i * bl, (i + 1) * bl)
        lg_b, mix_b = layer._prep(Q[:, :, sl], K[:, :, sl], V[:, :, sl], bl, a)
        lg[:, :, sl] = lg_b
        mix[:, :, sl] = mix_b
    sm_scale = (layer.d_head / layer.r) ** 0.5
    Y, S_end = sharded_attention_core(Q, K, V, lg, mix, layer.r, sm_scale, layer.gla_scale, T, group=group,
                                      log_alpha=layer.log_alpha if layer.learnable_alpha else None)
    out = layer._out(Y, B, Tl, dtype_in)
    return (out, S_end) if return_state else out


def shard_tokens(x: torch.Tensor, world: int, rank: int, dim: int = 1) -> torch.Tensor:
    """This rank's tokens of a full-sequence tensor (its two zig-zag blocks,
    concatenated along ``dim``)."""
    T = x.shape[dim]
    return torch.cat([x.narrow(dim, a, e - a) for a, e in zigzag_blocks(T, world, rank)], dim=dim)
