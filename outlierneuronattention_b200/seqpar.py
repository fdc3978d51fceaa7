"""Sequence-sharded prefill of the HOFA attention core (long contexts over N GPUs),
and the hand-over of its caches to head-sharded decode.

A long prompt is cut into 2N equal blocks and rank r owns blocks r and
2N-1-r ("zig-zag"), so that every rank gets the same amount of causal
attention work.  One exchange step per layer, one process per GPU over
``torch.distributed`` (NCCL on GPUs):

* outlier attention: query block i needs the rotated outlier keys K_O and the
  values V of blocks 0..i.  Every rank keeps one full-sequence key|value
  buffer in token-major layout ``[T, B, H, r + D]``, where any block is one
  contiguous range.  Its own blocks are copied in; every block another rank
  needs lands straight in the receiver's buffer at the block's sequence
  position: block r goes to every other rank (one in-place all-gather of the
  first-half blocks), block 2N-1-r to the ranks below r (NCCL ``isend`` /
  ``irecv`` in one batch).  The
  transfers run on NCCL's stream while the first GLA pass runs; then the
  attention of each local block reads the key prefix ending at its last token
  (``q_offset`` = the block's first absolute position), the two blocks on two
  side streams, while the block-state exchange and the second GLA pass run on
  the caller's stream underneath them;
* GLA: both local blocks run from a zero state in one call (the blocks are a
  batch of two), giving their end states S_b and total log decays G_b.  These
  are all-gathered, and every rank forms the start state of each of its blocks
  from all earlier blocks at once,
  ``S_in[i] = sum_{k<i} exp(c_i - c_{k+1}) S_k`` with ``c`` the exclusive
  prefix sum of the block decays (the reference's carried-state recurrence,
  src/chunk_gla_inlier.py:86-126, unrolled over blocks; every exponent is a
  sum of log decays and so <= 0).  The blocks are then run again from their
  start states with the fused ``(1-mix) * gla_scale * RMSNorm`` epilogue
  (RMSNorm is not linear, so the normalised output has to wait for the start
  state);
* the attention output (mix * attention, in a buffer of its own) is then
  added into the GLA output (as in the layer, two roundings).

``relayout_seq_to_head`` turns the sequence-sharded result into the caches of
a head-sharded decode: rank g ends up with the outlier key and value caches
of every token for its head range (one ``all_to_all_single``) and its heads'
rows of the final GLA state (identical on every rank after the prefill).

The compute functions default to this library's CUDA operators
(``gla_forward`` and ``exact_attention_triton``); they are parameters so that
the exchange logic can be checked on CPU ranks against another implementation
of the same operators.
"""
from __future__ import annotations

from typing import Callable, Dict, List, Optional, Tuple

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


def block_receivers(i: int, world: int) -> List[int]:
    """Ranks other than the owner that need global block ``i``'s keys: every
    rank owning a later block (its second block 2N-1-s is later than i)."""
    owner, _ = block_owner(i, world)
    return [s for s in range(world) if s != owner and 2 * world - 1 - s > i]


def head_range(H: int, world: int, rank: int) -> Tuple[int, int]:
    """[h0, h1) heads of ``rank`` when H heads are split evenly over the ranks."""
    if H % world != 0:
        raise ValueError(f"{H} heads do not split evenly over {world} ranks")
    hg = H // world
    return rank * hg, (rank + 1) * hg


def _group_info(group) -> Tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def _global_rank(group, r: int) -> int:
    return r if group is None else dist.get_global_rank(group, r)


class PhaseTimer:
    """CUDA events at the phase boundaries of ``sharded_attention_core`` (on
    the current stream); ``ms()`` after a synchronisation gives the time of
    each phase."""

    def __init__(self):
        self.events: List[Tuple[str, torch.cuda.Event]] = []

    def mark(self, name: str):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self.events.append((name, e))

    def ms(self) -> Dict[str, float]:
        out = {}
        for (_, a), (name, b) in zip(self.events, self.events[1:]):
            out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        return out


_SIDE_STREAMS: Dict[int, Tuple[torch.cuda.Stream, torch.cuda.Stream]] = {}


def _side_streams(dev: torch.device):
    """Two extra streams per device for the attention launches of the two
    local blocks (concurrent with each other and with the GLA on the current
    stream)."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    st = _SIDE_STREAMS.get(idx)
    if st is None:
        d = torch.device("cuda", idx)
        st = _SIDE_STREAMS[idx] = (torch.cuda.Stream(d), torch.cuda.Stream(d))
    return st


def _as_block_batch(x: torch.Tensor, bl: int) -> Optional[torch.Tensor]:
    """[B, H, 2*bl, ...] -> [2*B, H, bl, ...] as a view (block-major batch),
    or None when the strides do not allow a view."""
    B = x.shape[0]
    y = x.unflatten(2, (2, bl)).movedim(2, 0)          # [2, B, H, bl, ...]
    try:
        return y.view(2 * B, *y.shape[2:])
    except RuntimeError:
        return None


def _block_prefix_states(S_blocks: torch.Tensor, G_blocks: torch.Tensor, want: List[int]) -> torch.Tensor:
    """Start states of the blocks in ``want`` (an index equal to the number of
    blocks asks for the state after the last block).

    S_blocks [n, B, H, J, D]: each block's end state from a zero start;
    G_blocks [n, B, H] or [n, B, H, J]: each block's total log decay (per
    channel with a per-channel decay).  ``S_in[i] = sum_{k<i} exp(c_i -
    c_{k+1}) S_k`` with ``c`` the exclusive prefix sum of G."""
    n = S_blocks.shape[0]
    c = torch.cat([torch.zeros_like(G_blocks[:1]), torch.cumsum(G_blocks, 0)], 0)     # [n+1, ...]
    # weights [w, n, ...]: exp(c_i - c_{k+1}) for k < i, else 0 (built from host
    # integers only: no host <-> device copy, so nothing here waits for the GPU)
    k = torch.arange(n, device=S_blocks.device).view(n, *([1] * (G_blocks.dim() - 1)))
    w = torch.stack([torch.where(k < i, torch.exp(torch.clamp(c[i] - c[1:], max=0.0)), 0.0) for i in want])
    if G_blocks.dim() == 3:                       # scalar decay per (b, h)
        return torch.einsum("wkbh,kbhjd->wbhjd", w, S_blocks)
    return torch.einsum("wkbhj,kbhjd->wbhjd", w, S_blocks)


def sharded_attention_core(Q, K, V, log_gamma, mix, r: int, sm_scale: float, gla_scale, T: int, *,
                           group=None, log_alpha=None, eps: float = FP32_EPS,
                           gla: Callable = gla_forward, attn: Callable = exact_attention_triton,
                           timer: Optional[PhaseTimer] = None, return_kv: bool = False):
    """The attention core of one rank of a sequence-sharded prefill.

    Q, K, V: [B,H,Tl,D] this rank's tokens (its two zig-zag blocks, in order,
    concatenated along T; Tl = T / world), with RoPE already applied to the
    first r channels of Q and K at the tokens' absolute positions;
    log_gamma [B,H,Tl] float32 and mix [B,H,Tl] (as produced by the layer's
    gate step); gla_scale [1,H,1,D]; T the whole sequence length.
    Returns (Y [B,H,Tl,D] for this rank's tokens, S_end [B,H,D-r,D] float32:
    the GLA state after all T tokens, identical on every rank); with
    ``return_kv`` also the full-sequence key/value buffers (token-major
    [T,B,H,r] and [T,B,H,D]; rows of blocks this rank did not need are
    unspecified; views of one [T,B,H,r+D] buffer).
    """
    world, rank = _group_info(group)
    B, H, Tl, D = Q.shape
    J = D - r
    nb = 2 * world
    blocks = zigzag_blocks(T, world, rank)
    bl = T // nb
    if Tl != 2 * bl:
        raise ValueError(f"rank holds {Tl} tokens, expected 2 blocks of {bl}")
    local = [slice(0, bl), slice(bl, 2 * bl)]
    dev, dt = Q.device, Q.dtype
    mark = timer.mark if timer is not None else (lambda name: None)
    mark("start")

    # 1. one full-sequence key|value buffer (token-major [T, B, H, r + D]: a
    #    block is one contiguous range), own blocks copied in, the exchange
    #    started: the first-half blocks (block s belongs to rank s, and every
    #    rank needs it) with one in-place all-gather into [0, N*bl), the
    #    second-half blocks point-to-point (block 2N-1-s goes to the ranks
    #    below s)
    C = r + D
    KVB = torch.empty(T, B, H, C, dtype=dt, device=dev)
    for (a, e), sl in zip(blocks, local):
        KVB[a:e, ..., :r].copy_(K[:, :, sl, :r].permute(2, 0, 1, 3))
        KVB[a:e, ..., r:].copy_(V[:, :, sl].permute(2, 0, 1, 3))
    works = []
    if world > 1:
        first = KVB[:world * bl]
        works.append(dist.all_gather_into_tensor(first, KVB[rank * bl:(rank + 1) * bl], group=group, async_op=True))
        ops = []
        for s_ in range(world):
            i = nb - 1 - s_                      # rank s_'s second block
            a, e = i * bl, (i + 1) * bl
            if s_ == rank:
                ops += [dist.P2POp(dist.isend, KVB[a:e], _global_rank(group, d), group) for d in range(rank)]
            elif rank < s_:
                ops.append(dist.P2POp(dist.irecv, KVB[a:e], _global_rank(group, s_), group))
        if ops:
            works += dist.batch_isend_irecv(ops)
    mark("pack_and_post")

    # 2. outlier attention of each local block against its key prefix, on two
    #    side streams that wait only for the key/value exchange (and, through
    #    it, the packing copies): it runs beside the GLA passes and the
    #    block-state exchange on this stream, into a buffer of its own
    #    (out = mix * attention)
    Kv = KVB[..., :r].permute(1, 2, 0, 3)           # [B, H, T, r] view
    Vv = KVB[..., r:].permute(1, 2, 0, 3)           # [B, H, T, D] view
    Ya = torch.empty(B, H, Tl, D, dtype=dt, device=dev)
    calls = [(Q[:, :, sl], e, a, sl) for (a, e), sl in zip(blocks, local)]
    sides = _side_streams(dev) if Q.is_cuda else None
    if sides is not None:
        cur = torch.cuda.current_stream(dev)
        for st, (q_, e, a, sl) in zip(sides, calls):
            st.wait_stream(cur)
            with torch.cuda.stream(st):
                for w in works:
                    w.wait()
                attn(q_, Kv[:, :, :e], Vv[:, :, :e], r, sm_scale, mix[:, :, sl], out=Ya[:, :, sl], q_offset=a,
                     accumulate=False)
    else:
        for w in works:
            w.wait()
        for q_, e, a, sl in calls:
            attn(q_, Kv[:, :, :e], Vv[:, :, :e], r, sm_scale, mix[:, :, sl], out=Ya[:, :, sl], q_offset=a,
                 accumulate=False)
    mark("attention_issued")

    # 3. GLA from a zero state for both local blocks (one call, a batch of two blocks)
    Qb, Kb, Vb = (_as_block_batch(x, bl) for x in (Q, K, V))
    lgb, mixb = _as_block_batch(log_gamma, bl), _as_block_batch(mix, bl)
    batched = all(x is not None for x in (Qb, Kb, Vb, lgb, mixb))
    S_loc = torch.empty(2 * B, H, J, D, dtype=torch.float32, device=dev)
    scratch = torch.empty(2 * B, H, bl, D, dtype=dt, device=dev)
    if batched:
        gla(Qb, Kb, Vb, lgb, r, log_alpha=log_alpha, y=scratch, state_out=S_loc, eps=eps)
    else:
        for i, sl in enumerate(local):
            gla(Q[:, :, sl], K[:, :, sl], V[:, :, sl], log_gamma[:, :, sl], r, log_alpha=log_alpha,
                y=scratch[i * B:(i + 1) * B], state_out=S_loc[i * B:(i + 1) * B], eps=eps)
    G_loc = log_gamma.float().unflatten(2, (2, bl)).sum(-1).movedim(2, 0).reshape(2 * B, H)   # [2B, H]
    if log_alpha is not None:
        G_loc = G_loc[..., None] * torch.exp(log_alpha.float().reshape(1, H, J))             # [2B, H, J]
    #    and the block-state exchange
    if world > 1:
        S_all = torch.empty(world * S_loc.shape[0], *S_loc.shape[1:], dtype=S_loc.dtype, device=dev)
        G_all = torch.empty(world * G_loc.shape[0], *G_loc.shape[1:], dtype=G_loc.dtype, device=dev)
        state_works = [dist.all_gather_into_tensor(S_all, S_loc.contiguous(), group=group, async_op=True),
                       dist.all_gather_into_tensor(G_all, G_loc.contiguous(), group=group, async_op=True)]
    else:
        S_all, G_all, state_works = S_loc, G_loc, []
    mark("gla_pass1")

    # 4. start states of the local blocks (and the end state) from every rank's block states
    for w in state_works:
        w.wait()
    S_all, G_all = S_all.view(world, *S_loc.shape), G_all.view(world, *G_loc.shape)
    order = [block_owner(i, world) for i in range(nb)]
    S_blocks = torch.stack([S_all[o][li * B:(li + 1) * B] for o, li in order])    # [nb, B, H, J, D]
    G_blocks = torch.stack([G_all[o][li * B:(li + 1) * B] for o, li in order])    # [nb, B, H(, J)]
    with torch.autocast(dev.type, enabled=False):                                # float32 state arithmetic
        starts = _block_prefix_states(S_blocks, G_blocks, [blocks[0][0] // bl, blocks[1][0] // bl, nb])
    S_end = starts[2]

    # 5. GLA again from each local block's start state, fused epilogue
    Y = torch.empty(B, H, Tl, D, dtype=dt, device=dev)
    Yb = _as_block_batch(Y, bl)
    if batched and Yb is not None:
        gla(Qb, Kb, Vb, lgb, r, log_alpha=log_alpha, mix_g=mixb, gla_scale=gla_scale, y=Yb,
            initial_state=starts[:2].reshape(2 * B, H, J, D), eps=eps)
    else:
        for i, sl in enumerate(local):
            gla(Q[:, :, sl], K[:, :, sl], V[:, :, sl], log_gamma[:, :, sl], r, log_alpha=log_alpha,
                mix_g=mix[:, :, sl], gla_scale=gla_scale, y=Y[:, :, sl], initial_state=starts[i].contiguous(),
                eps=eps)
    mark("state_exchange_gla_pass2")

    # 6. the attention output joins the GLA output (as in the layer)
    if sides is not None:
        for st in sides:
            torch.cuda.current_stream(dev).wait_stream(st)
    mark("attention_end")
    Y.add_(Ya)
    mark("add")
    if return_kv:
        return Y, S_end, (KVB[..., :r], KVB[..., r:])
    return Y, S_end


def relayout_seq_to_head(K_loc: torch.Tensor, V_loc: torch.Tensor, S_end: torch.Tensor, T: int, capacity: int,
                         group=None):
    """Caches of a head-sharded decode from a sequence-sharded prefill.

    K_loc [B,H,Tl,>=r] (rotated outlier keys, channels [0, r) used) and V_loc
    [B,H,Tl,D]: this rank's two zig-zag blocks; r = the caller's key width
    (``K_loc.shape[3]``); S_end [B,H,J,D] the GLA state after all T tokens
    (identical on every rank).  Rank g gets heads ``head_range(H, world, g)``:
    returns (cache_k [B,Hg,capacity,r], cache_v [B,Hg,capacity,D],
    state [B,Hg,J,D]) with rows [0, T) filled in sequence order (rows
    [T, capacity) are left for the decode steps).  One ``all_to_all_single``
    moves every rank's blocks of head group g to rank g."""
    world, rank = _group_info(group)
    B, H, Tl, r = K_loc.shape
    D = V_loc.shape[3]
    h0, h1 = head_range(H, world, rank)
    Hg = h1 - h0
    nb, bl = 2 * world, T // (2 * world)
    if capacity < T:
        raise ValueError(f"cache capacity {capacity} below the prompt length {T}")
    C = r + D
    # send[g] = this rank's two blocks of head group g, [2, B, Hg, bl, C]
    send = torch.empty(world, 2, B, Hg, bl, C, dtype=K_loc.dtype, device=K_loc.device)
    for g in range(world):
        a, e = g * Hg, (g + 1) * Hg
        for li in range(2):
            sl = slice(li * bl, (li + 1) * bl)
            send[g, li, ..., :r].copy_(K_loc[:, a:e, sl])
            send[g, li, ..., r:].copy_(V_loc[:, a:e, sl])
    recv = torch.empty_like(send)
    if world > 1:
        dist.all_to_all_single(recv, send, group=group)
    else:
        recv.copy_(send)
    cache_k = torch.empty(B, Hg, capacity, r, dtype=K_loc.dtype, device=K_loc.device)
    cache_v = torch.empty(B, Hg, capacity, D, dtype=V_loc.dtype, device=V_loc.device)
    for i in range(nb):
        src, li = block_owner(i, world)
        cache_k[:, :, i * bl:(i + 1) * bl].copy_(recv[src, li, ..., :r])
        cache_v[:, :, i * bl:(i + 1) * bl].copy_(recv[src, li, ..., r:])
    return cache_k, cache_v, S_end[:, h0:h1].contiguous()


def sharded_layer_forward(layer, x_local: torch.Tensor, T: int, group=None, return_state: bool = False):
    """Prefill of a ``HybridOutlierFactorizedAttention`` layer with the
    sequence sharded over the ranks of ``group``.

    x_local: [B, T/world, d_model], this rank's tokens (its two zig-zag blocks
    concatenated); T the whole sequence length.  Returns this rank's rows of
    the layer output ([B, T/world, d_model]), and with ``return_state`` also
    the GLA state after all T tokens (every rank holds it) and this rank's
    rotated outlier keys and values ([B,H,T/world,r], [B,H,T/world,d_head],
    the input of ``relayout_seq_to_head``).  Hybrid layers only
    (0 < r < d_head, no width split)."""
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
                                      log_alpha=layer.log_alpha if layer.learnable_alpha else None,
                                      eps=layer.hybrid_prefill_eps)
    out = layer._out(Y, B, Tl, dtype_in)
    if return_state:
        return out, S_end, (K[..., :layer.r], V)
    return out


def shard_tokens(x: torch.Tensor, world: int, rank: int, dim: int = 1) -> torch.Tensor:
    """This rank's tokens of a full-sequence tensor (its two zig-zag blocks,
    concatenated along ``dim``)."""
    T = x.shape[dim]
    return torch.cat([x.narrow(dim, a, e - a) for a, e in zigzag_blocks(T, world, rank)], dim=dim)
