"""Parity of the fused decode kernel (hofa_decode_fwd via fused_hofa_decode)
against the CPU oracle ``decode_core`` (restating src/hofa_decode_triton.py:
342-476) on identical seeded inputs.

Tolerances: outputs in bf16/fp16 <= 2e-2 max-abs; float32 inputs <= 1e-4;
the float32 GLA state <= 1e-5 abs (+1e-5 rel) in every dtype.
"""
import math

import pytest
import torch
import torch.nn.functional as F

from oracle.hofa_oracle import FP32_EPS, decode_core

pytestmark = pytest.mark.gpu

TOL = {torch.bfloat16: 2e-2, torch.float16: 2e-2, torch.float32: 1e-4}


def make_inputs(B, H, D, R, L, dtype, seed, alpha=False, cache_stride_pad=0):
    g = torch.Generator().manual_seed(seed)
    J = D - R
    rn = lambda *s: torch.randn(*s, generator=g)
    q, k, v = rn(B, H, 1, D), rn(B, H, 1, D), rn(B, H, 1, D)
    Rw = R + cache_stride_pad
    ck_full = rn(B, H, L, max(Rw, 1))
    cache_k = ck_full[..., :R]
    cache_v = rn(B, H, L, D)
    state = rn(B, H, J, D) * 0.1
    log_gamma = F.logsigmoid(rn(B, H, 1) * 2.0)
    mix = torch.sigmoid(rn(B, H, 1))
    norm_w = 1.0 + 0.2 * rn(H, D)
    log_alpha = rn(1, H, 1, J) * 0.5 if alpha else None
    dev = lambda t, dt=dtype: None if t is None else t.to(dt).cuda()
    gpu = dict(q=dev(q), k=dev(k), v=dev(v), cache_k=dev(ck_full)[..., :R] if cache_stride_pad else dev(cache_k),
               cache_v=dev(cache_v), state_in=state.cuda(), log_gamma=log_gamma.cuda(), mix_g=dev(mix),
               norm_w=norm_w.cuda(), log_alpha=dev(log_alpha, torch.float32))
    # the oracle sees exactly the (rounded) values the kernel sees
    cpu = {k_: (None if t is None else t.detach().cpu()) for k_, t in gpu.items()}
    return gpu, cpu


def run_pair(B, H, D, R, L, seq_len, dtype, seed=0, split_k=None, alpha=False, cache_stride_pad=0):
    from outlierneuronattention_b200 import fused_hofa_decode
    gpu, cpu = make_inputs(B, H, D, R, L, dtype, seed, alpha, cache_stride_pad)
    sm_scale = math.sqrt(D / R) if R else 1.0
    state_out = torch.empty_like(gpu["state_in"])
    y = fused_hofa_decode(gpu["q"], gpu["k"], gpu["v"], gpu["cache_k"], gpu["cache_v"], gpu["state_in"], state_out,
                          gpu["log_gamma"], gpu["mix_g"], gpu["norm_w"], R, seq_len, sm_scale, split_k=split_k,
                          log_alpha=gpu["log_alpha"])
    torch.cuda.synchronize()
    y_ref, s_ref = decode_core(cpu["q"], cpu["k"], cpu["v"], cpu["cache_k"], cpu["cache_v"], cpu["state_in"],
                               cpu["log_gamma"], cpu["mix_g"], cpu["norm_w"], R, seq_len, sm_scale,
                               log_alpha=cpu["log_alpha"], eps=FP32_EPS)
    return y, state_out, y_ref, s_ref


def check(y, s, y_ref, s_ref, dtype):
    assert y.dtype == dtype
    err = (y.double().cpu() - y_ref).abs().max().item()
    assert err <= TOL[dtype], f"max-abs {err}"
    torch.testing.assert_close(s.double().cpu(), s_ref, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("B", [1, 2, 4])
def test_config1_decode_bf16(B):
    """d_model=1024 -> H=16, d_h=64, r=16, L=4096."""
    check(*run_pair(B, 16, 64, 16, 4096, 4096, torch.bfloat16, seed=B), torch.bfloat16)


@pytest.mark.parametrize("R", [88, 96])
def test_fp32_large_r_without_room_for_the_ring(R):
    """float32 at head dim 128 with most channels in the outlier path: even a
    4-stage ring of 64-token chunks would need more shared memory than a CTA
    gets (4 x 64 x (R + 128) x 4 bytes), so the launcher takes the 16-byte
    register-load path; it still matches the oracle."""
    check(*run_pair(1, 2, 128, R, 300, 300, torch.float32, seed=R), torch.float32)


@pytest.mark.parametrize("split_k", [1, 2, 3, 6, 7, 12, 64])
def test_split_counts(split_k):
    check(*run_pair(2, 4, 64, 16, 1000, 1000, torch.bfloat16, seed=10 + split_k, split_k=split_k), torch.bfloat16)


@pytest.mark.parametrize("seq_len", [1, 2, 31, 32, 33, 129])
def test_ragged_lengths_read_only_the_prefix(seq_len):
    """Rows >= seq_len of a pre-allocated cache hold NaN and must not be read."""
    from outlierneuronattention_b200 import fused_hofa_decode
    gpu, cpu = make_inputs(2, 3, 64, 16, 256, torch.bfloat16, seed=seq_len)
    gpu["cache_k"][:, :, seq_len:] = float("nan")
    gpu["cache_v"][:, :, seq_len:] = float("nan")
    out = torch.empty_like(gpu["state_in"])
    for split in (None, 5):
        y = fused_hofa_decode(gpu["q"], gpu["k"], gpu["v"], gpu["cache_k"], gpu["cache_v"], gpu["state_in"], out,
                              gpu["log_gamma"], gpu["mix_g"], gpu["norm_w"], 16, seq_len, 2.0, split_k=split)
        y_ref, s_ref = decode_core(cpu["q"], cpu["k"], cpu["v"], cpu["cache_k"], cpu["cache_v"], cpu["state_in"],
                                   cpu["log_gamma"], cpu["mix_g"], cpu["norm_w"], 16, seq_len, 2.0)
        assert torch.isfinite(y).all()
        check(y, out, y_ref, s_ref, torch.bfloat16)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_dtypes(dtype):
    check(*run_pair(2, 4, 64, 16, 700, 650, dtype, seed=3), dtype)


@pytest.mark.parametrize("D,R", [(128, 16), (128, 32), (128, 64), (32, 8), (64, 32), (64, 8)])
def test_head_dims_and_outlier_widths(D, R):
    check(*run_pair(2, 2, D, R, 300, 300, torch.bfloat16, seed=D + R), torch.bfloat16)


def test_learnable_alpha():
    check(*run_pair(2, 4, 64, 16, 400, 399, torch.bfloat16, seed=5, alpha=True), torch.bfloat16)


def test_generic_strided_cache_path():
    """A cache whose rows are not 16-byte aligned takes the scalar-load path."""
    check(*run_pair(2, 3, 64, 16, 300, 300, torch.bfloat16, seed=6, cache_stride_pad=4), torch.bfloat16)
    check(*run_pair(2, 3, 64, 12, 300, 300, torch.bfloat16, seed=7), torch.bfloat16)  # R not a multiple of 8


def test_r0_is_gla_only():
    check(*run_pair(2, 4, 64, 0, 1, 1, torch.bfloat16, seed=8), torch.bfloat16)


def test_repeated_launches_rearm_the_workspace():
    from outlierneuronattention_b200 import fused_hofa_decode
    gpu, _ = make_inputs(4, 16, 64, 16, 2048, torch.bfloat16, seed=9)
    out = torch.empty_like(gpu["state_in"])
    ys = [fused_hofa_decode(gpu["q"], gpu["k"], gpu["v"], gpu["cache_k"], gpu["cache_v"], gpu["state_in"], out,
                            gpu["log_gamma"], gpu["mix_g"], gpu["norm_w"], 16, 2048, 2.0, split_k=8) for _ in range(5)]
    for y in ys[1:]:
        assert torch.equal(y, ys[0])


def test_device_seq_len_and_graph_replay():
    """seq_len from device memory, captured once in a CUDA graph, replayed
    with different lengths; an out-of-range length is clamped and flagged."""
    from outlierneuronattention_b200 import fused_hofa_decode
    from outlierneuronattention_b200.hofa_decode import read_status
    B, H, D, R, L = 2, 4, 64, 16, 512
    gpu, cpu = make_inputs(B, H, D, R, L, torch.bfloat16, seed=11)
    out = torch.empty_like(gpu["state_in"])
    sl = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    args = (gpu["q"], gpu["k"], gpu["v"], gpu["cache_k"], gpu["cache_v"], gpu["state_in"], out,
            gpu["log_gamma"], gpu["mix_g"], gpu["norm_w"], R, L, 2.0)
    fused_hofa_decode(*args, split_k=4, seq_len_dev=sl)  # warm-up outside capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y_static = fused_hofa_decode(*args, split_k=4, seq_len_dev=sl)
    for n in (1, 100, 512):
        sl.fill_(n)
        graph.replay()
        torch.cuda.synchronize()
        y_ref, s_ref = decode_core(cpu["q"], cpu["k"], cpu["v"], cpu["cache_k"], cpu["cache_v"], cpu["state_in"],
                                   cpu["log_gamma"], cpu["mix_g"], cpu["norm_w"], R, n, 2.0)
        check(y_static, out, y_ref, s_ref, torch.bfloat16)
    assert read_status(gpu["q"].device, B, H, D) == 0
    sl.fill_(L + 5)
    graph.replay()
    torch.cuda.synchronize()
    assert read_status(gpu["q"].device, B, H, D) == 1
    assert read_status(gpu["q"].device, B, H, D) == 0  # reading clears the word
    y_ref, _ = decode_core(cpu["q"], cpu["k"], cpu["v"], cpu["cache_k"], cpu["cache_v"], cpu["state_in"],
                           cpu["log_gamma"], cpu["mix_g"], cpu["norm_w"], R, L, 2.0)
    assert (y_static.double().cpu() - y_ref).abs().max().item() <= 2e-2


def test_broadcast_mix_and_bf16_log_gamma():
    """fixed-blend mix is an expanded [1,H,1] view (batch stride 0); log_gamma
    may arrive in the activation dtype."""
    from outlierneuronattention_b200 import fused_hofa_decode
    gpu, cpu = make_inputs(3, 4, 64, 16, 200, torch.bfloat16, seed=12)
    mix = torch.sigmoid(torch.randn(1, 4, 1, generator=torch.Generator().manual_seed(167))).to(torch.bfloat16)
    lg = gpu["log_gamma"].to(torch.bfloat16)
    out = torch.empty_like(gpu["state_in"])
    y = fused_hofa_decode(gpu["q"], gpu["k"], gpu["v"], gpu["cache_k"], gpu["cache_v"], gpu["state_in"], out,
                          lg, mix.cuda().expand(3, 4, 1), gpu["norm_w"], 16, 200, 2.0)
    y_ref, s_ref = decode_core(cpu["q"], cpu["k"], cpu["v"], cpu["cache_k"], cpu["cache_v"], cpu["state_in"],
                               lg.cpu(), mix.expand(3, 4, 1), cpu["norm_w"], 16, 200, 2.0)
    check(y, out, y_ref, s_ref, torch.bfloat16)


def test_cpu_tensors_are_rejected():
    from outlierneuronattention_b200 import fused_hofa_decode
    gpu, cpu = make_inputs(1, 2, 64, 16, 8, torch.bfloat16, seed=13)
    with pytest.raises(ValueError, match="CUDA"):
        fused_hofa_decode(cpu["q"], cpu["k"], cpu["v"], cpu["cache_k"], cpu["cache_v"], cpu["state_in"],
                          torch.empty_like(cpu["state_in"]), cpu["log_gamma"], cpu["mix_g"], cpu["norm_w"], 16, 8, 2.0)
