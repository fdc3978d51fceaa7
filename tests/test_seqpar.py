"""Sequence-sharded prefill (outlierneuronattention_b200.seqpar).

CPU tests run the exchange logic on gloo ranks (world sizes 2, 3 and 4) with
the oracle's GLA and attention as the compute functions, and compare every
rank's rows with the oracle's whole-sequence result; the seq -> head re-layout
is checked the same way against the whole-sequence caches.  The GPU tests run
the layer through the CUDA path with one rank and two zig-zag blocks (initial
states, key prefixes with q_offset, RoPE at block offsets) against the layer's
own single-pass forward, and with two ranks over NCCL when two GPUs are there.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from outlierneuronattention_b200 import seqpar
from oracle.hofa_oracle import chunk_gla_core, outlier_attention_core


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# ---- the oracle as compute functions with the CUDA operators' signatures ----
def oracle_gla(Q, K, V, log_gamma, r, *, log_alpha=None, mix_g=None, gla_scale=None, y=None, state_out=None,
               initial_state=None, eps=1e-5):
    yy, S = chunk_gla_core(Q, K, V, log_gamma, r, log_alpha=log_alpha, mix_g=mix_g, gla_scale=gla_scale,
                           eps=eps, state_init=initial_state)
    if y is not None:
        y.copy_(yy)
    if state_out is not None:
        state_out.copy_(S)
    return y


def oracle_attn(q, k, v, r, sm_scale, mix_g, out=None, q_offset=0, accumulate=True):
    res = outlier_attention_core(q, k, v, r, sm_scale, mix_g, out=out if accumulate else None, q_offset=q_offset)
    out.copy_(res)
    return out


def _inputs(B, H, T, D, r, alpha, seed=0):
    g = torch.Generator().manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)
    Q, K, V = rn(B, H, T, D), rn(B, H, T, D), rn(B, H, T, D)
    lg = torch.nn.functional.logsigmoid(rn(B, H, T) + 2.0)
    mix = torch.sigmoid(rn(B, H, T))
    gs = 1 + 0.1 * rn(1, H, 1, D)
    la = 0.3 * rn(1, H, 1, D - r) if alpha else None
    return Q, K, V, lg, mix, gs, la


def _full(Q, K, V, lg, mix, gs, la, r, sm_scale):
    Y, S = chunk_gla_core(Q, K, V, lg, r, log_alpha=la, mix_g=mix, gla_scale=gs, eps=1e-6)
    Y = outlier_attention_core(Q, K, V, r, sm_scale, mix, out=Y)
    return Y, S


def _rank_main(rank, world, port, alpha, B):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", world_size=world, rank=rank)
    try:
        H, T, D, r = 2 * world, 24 * world, 16, 4
        Q, K, V, lg, mix, gs, la = _inputs(B, H, T, D, r, alpha)
        sm = 2.0
        Y_ref, S_ref = _full(Q, K, V, lg, mix, gs, la, r, sm)
        take = lambda x: seqpar.shard_tokens(x, world, rank, dim=2)
        Y, S_end, (KB, VB) = seqpar.sharded_attention_core(take(Q), take(K), take(V), take(lg), take(mix), r, sm, gs,
                                                           T, log_alpha=la, eps=1e-6, gla=oracle_gla,
                                                           attn=oracle_attn, return_kv=True)
        # the state crosses ranks in float32, as in the CUDA path
        assert (Y - take(Y_ref)).abs().max().item() < 1e-5
        assert (S_end.double() - S_ref).abs().max().item() < 1e-5
        # every key block this rank attends to arrived at its sequence position
        last = seqpar.zigzag_blocks(T, world, rank)[1][1]
        assert torch.equal(KB[:last].permute(1, 2, 0, 3), K[:, :, :last, :r])
        assert torch.equal(VB[:last].permute(1, 2, 0, 3), V[:, :, :last])
        # seq -> head re-layout for a head-sharded decode
        ck, cv, st = seqpar.relayout_seq_to_head(take(K)[..., :r], take(V), S_end, T, T + 5)
        h0, h1 = seqpar.head_range(H, world, rank)
        assert ck.shape == (B, h1 - h0, T + 5, r) and cv.shape == (B, h1 - h0, T + 5, D)
        assert torch.equal(ck[:, :, :T], K[:, h0:h1, :, :r]) and torch.equal(cv[:, :, :T], V[:, h0:h1])
        assert torch.equal(st, S_end[:, h0:h1])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,alpha,B", [(2, False, 1), (3, False, 1), (2, True, 1), (4, False, 1), (2, False, 2)])
def test_sharded_core_matches_whole_sequence_on_gloo_ranks(world, alpha, B):
    """B = 2 takes the per-block GLA calls (the two blocks are not a batch view)."""
    mp.start_processes(_rank_main, args=(world, _free_port(), alpha, B), nprocs=world, join=True,
                       start_method="spawn")


def test_block_receivers_cover_every_causal_need():
    for world in (1, 2, 3, 8):
        nb = 2 * world
        for s in range(world):
            own = {s, nb - 1 - s}
            need = {i for i in range(nb - 1 - s) if i not in own}   # blocks before its second block
            got = {i for i in range(nb) if s in seqpar.block_receivers(i, world)}
            assert got == need, (world, s)


def test_block_prefix_states_match_the_recurrence():
    g = torch.Generator().manual_seed(5)
    n, B, H, J, D = 6, 2, 3, 4, 5
    S = torch.randn(n, B, H, J, D, generator=g, dtype=torch.float64)
    for G in (-torch.rand(n, B, H, generator=g, dtype=torch.float64) * 3,
              -torch.rand(n, B, H, J, generator=g, dtype=torch.float64) * 3):
        run, ref = torch.zeros(B, H, J, D, dtype=torch.float64), []
        for i in range(n):
            ref.append(run)
            dec = torch.exp(G[i])
            run = (dec[..., None, None] if G.dim() == 3 else dec[..., None]) * run + S[i]
        ref.append(run)
        got = seqpar._block_prefix_states(S, G, list(range(n + 1)))
        assert torch.allclose(got, torch.stack(ref), atol=1e-12)


def test_zigzag_blocks_partition_and_balance():
    T, world = 96, 4
    owned = sorted(b for r in range(world) for b in seqpar.zigzag_blocks(T, world, r))
    assert owned == [(i * 12, (i + 1) * 12) for i in range(8)]
    # causal work of a block of queries [a, e): sum over its rows of (row + 1) keys
    work = [sum(sum(range(a + 1, e + 1)) for a, e in seqpar.zigzag_blocks(T, world, r)) for r in range(world)]
    assert max(work) == min(work)
    x = torch.arange(T).view(1, T)
    assert seqpar.shard_tokens(x, world, 1).tolist() == [list(range(12, 24)) + list(range(72, 84))]
    with pytest.raises(ValueError):
        seqpar.zigzag_blocks(100, 4, 0)


def test_single_rank_two_blocks_on_cpu_oracle():
    """World of one (no process group): the two-block path alone."""
    B, H, T, D, r = 2, 2, 40, 16, 4
    Q, K, V, lg, mix, gs, la = _inputs(B, H, T, D, r, alpha=False, seed=3)
    Y_ref, S_ref = _full(Q, K, V, lg, mix, gs, la, r, 2.0)
    Y, S = seqpar.sharded_attention_core(Q, K, V, lg, mix, r, 2.0, gs, T, eps=1e-6, gla=oracle_gla,
                                         attn=oracle_attn)
    ck, cv, st = seqpar.relayout_seq_to_head(K[..., :r], V, S, T, T)
    assert torch.equal(ck, K[..., :r]) and torch.equal(cv, V) and torch.equal(st, S)
    assert (Y - Y_ref).abs().max().item() < 1e-5
    assert (S.double() - S_ref).abs().max().item() < 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,tol", [(torch.float32, 2e-4), (torch.bfloat16, 3e-2)])
def test_sharded_layer_forward_one_rank_matches_layer_forward(dtype, tol):
    from outlierneuronattention_b200 import HybridOutlierFactorizedAttention, ModelConfig
    torch.manual_seed(0)
    cfg = ModelConfig(d_model=256, num_heads=4, num_layers=1, r=16, chunk_size=64)
    layer = HybridOutlierFactorizedAttention(cfg).cuda()
    with torch.no_grad():
        for name, prm in layer.named_parameters():
            if "gate_proj" in name or "mix_proj" in name:
                prm.normal_(0, 0.02)
    T = 512
    x = torch.randn(1, T, 256, generator=torch.Generator().manual_seed(122)).cuda()
    with torch.no_grad(), torch.autocast("cuda", dtype=dtype, enabled=dtype != torch.float32):
        ref, _, (st_ref, _) = layer(x, return_state=True)
        out, st, _ = seqpar.sharded_layer_forward(layer, x, T, return_state=True)
    assert (out.float() - ref.float()).abs().max().item() <= tol
    assert (st - st_ref).abs().max().item() <= tol


def _nccl_rank(rank, world, port, result_dir):
    from datetime import timedelta
    from outlierneuronattention_b200 import HybridOutlierFactorizedAttention, ModelConfig
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", world_size=world, rank=rank,
                            timeout=timedelta(seconds=120))
    try:
        torch.manual_seed(0)
        cfg = ModelConfig(d_model=256, num_heads=4, num_layers=1, r=16, chunk_size=64)
        layer = HybridOutlierFactorizedAttention(cfg).cuda()
        with torch.no_grad():
            for name, prm in layer.named_parameters():
                if "gate_proj" in name or "mix_proj" in name:
                    prm.normal_(0, 0.02)
        T = 1024
        x = torch.randn(1, T, 256, generator=torch.Generator().manual_seed(1)).cuda()
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            ref, _, (st_ref, _) = layer(x, return_state=True)
            out, st, _ = seqpar.sharded_layer_forward(layer, seqpar.shard_tokens(x, world, rank), T,
                                                      return_state=True)
        err = (out.float() - seqpar.shard_tokens(ref, world, rank).float()).abs().max().item()
        serr = (st - st_ref).abs().max().item()
        with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
            f.write(f"{err} {serr}\n")
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_layer_forward_two_gpus_nccl(tmp_path):
    world = 2
    mp.start_processes(_nccl_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for rank in range(world):
        err, serr = map(float, open(tmp_path / f"rank{rank}.txt").read().split())
        assert err <= 3e-2 and serr <= 3e-2, (rank, err, serr)
