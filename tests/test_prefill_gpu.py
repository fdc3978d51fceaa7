"""Parity of the prefill kernels against the CPU oracle on identical seeded
inputs:

* hofa_prefill_gla_fwd (chunk_gla_inlier_fwd) vs ``chunk_gla_core``
  (restating src/chunk_gla_inlier.py:153-237);
* hofa_prefill_outlier_fwd (exact_attention_triton) vs
  ``outlier_attention_core`` (restating src/exact_attention.py:163-188).

Tolerances (absolute, max over all elements): bf16/fp16 outputs <= 2e-2;
float32 inputs <= 1e-4; the final float32 GLA state <= 2e-2 in bf16/fp16 runs
and <= 1e-4 in float32 runs.  Raw (un-normalised) GLA outputs are checked on
inputs scaled so that |y| stays below about 4, where a bf16 output's own
rounding is below 1e-2.  The full-size tests print the achieved max-abs
errors.
"""
import math

import pytest
import torch
import torch.nn.functional as F

from oracle.hofa_oracle import chunk_gla_core, outlier_attention_core

pytestmark = pytest.mark.gpu


def rand_qkv(B, H, T, D, dtype, seed, scale=0.5):
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(B, H, T, D, generator=g) * scale for _ in range(3))
    lg = F.logsigmoid(torch.randn(B, H, T, generator=g) * 2.0 + 1.0)
    mix = torch.sigmoid(torch.randn(B, H, T, generator=g))
    gs = 1.0 + 0.2 * torch.randn(1, H, 1, D, generator=g)
    cast = lambda t: t.to(dtype)
    return cast(q), cast(k), cast(v), lg, cast(mix), gs


def maxabs(a, b):
    return (a.double().cpu() - b.double()).abs().max().item()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("T", [1, 63, 64, 65, 200, 1000])
def test_gla_fused_epilogue(dtype, T):
    from outlierneuronattention_b200 import chunk_gla_inlier_fwd
    B, H, D, r = 2, 3, 64, 16
    q, k, v, lg, mix, gs = rand_qkv(B, H, T, D, dtype, seed=T)
    Y, st = chunk_gla_inlier_fwd(q.cuda(), k.cuda(), v.cuda(), lg.cuda(), r, 64, mix_g=mix.cuda(), gla_scale=gs.cuda())
    Yr, Sr = chunk_gla_core(q, k, v, lg, r, 64, mix_g=mix, gla_scale=gs, eps=1e-5)
    assert st.shape == (B, H, 64, 64)
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    assert maxabs(Y, Yr) <= tol
    assert maxabs(st[:, :, :D - r, :D], Sr) <= tol
    assert st[:, :, D - r:].abs().max().item() == 0


@pytest.mark.parametrize("nseg", [1, 2, 3, 7])
def test_gla_segments_and_initial_state(nseg):
    from outlierneuronattention_b200.chunk_gla_inlier import gla_forward
    B, H, T, D, r = 2, 2, 700, 64, 16
    q, k, v, lg, mix, gs = rand_qkv(B, H, T, D, torch.float32, seed=100 + nseg)
    s0 = torch.randn(B, H, D - r, D, generator=torch.Generator().manual_seed(61)) * 0.3
    st = torch.empty(B, H, D - r, D, device="cuda")
    Y = gla_forward(q.cuda(), k.cuda(), v.cuda(), lg.cuda(), r, mix_g=mix.cuda(), gla_scale=gs.cuda(),
                    state_out=st, initial_state=s0.cuda(), num_segments=nseg)
    Yr, Sr = chunk_gla_core(q, k, v, lg, r, 64, mix_g=mix, gla_scale=gs, eps=1e-5, state_init=s0)
    assert maxabs(Y, Yr) <= 1e-4
    assert maxabs(st, Sr) <= 1e-4


@pytest.mark.parametrize("D,r", [(128, 16), (128, 64), (32, 8), (64, 0), (64, 32)])
def test_gla_shapes_raw_output(D, r):
    from outlierneuronattention_b200 import chunk_gla_inlier_fwd
    B, H, T = 2, 2, 300
    q, k, v, lg, _, _ = rand_qkv(B, H, T, D, torch.bfloat16, seed=D * 7 + r, scale=0.3)
    Y, st = chunk_gla_inlier_fwd(q.cuda(), k.cuda(), v.cuda(), lg.cuda(), r, 64)
    Yr, Sr = chunk_gla_core(q, k, v, lg, r, 64)
    assert Yr.abs().max().item() < 4.0  # keeps the bf16 output's own rounding below 1e-2
    assert maxabs(Y, Yr) <= 2e-2
    assert maxabs(st[:, :, :D - r, :D], Sr) <= 2e-2


def test_gla_learnable_alpha_strong_decay():
    """Per-channel decay exponents with strong decay (factored forms overflow there)."""
    from outlierneuronattention_b200 import chunk_gla_inlier_fwd
    B, H, T, D, r = 1, 2, 256, 64, 16
    q, k, v, _, mix, gs = rand_qkv(B, H, T, D, torch.float32, seed=55)
    g = torch.Generator().manual_seed(56)  # inputs independent of the tests that ran before
    lg = F.logsigmoid(torch.randn(B, H, T, generator=g) * 2.0 - 3.0)  # gamma ~ 0.05
    la = torch.randn(1, H, 1, D - r, generator=g) * 0.5
    Y, st = chunk_gla_inlier_fwd(q.cuda(), k.cuda(), v.cuda(), lg.cuda(), r, 64, log_alpha=la.cuda(),
                                 mix_g=mix.cuda(), gla_scale=gs.cuda())
    Yr, Sr = chunk_gla_core(q, k, v, lg, r, 64, log_alpha=la, mix_g=mix, gla_scale=gs, eps=1e-5)
    assert torch.isfinite(Y).all()
    # strong decay keeps the pre-norm output small and RMSNorm scales its fp32
    # rounding up with it: bound the error relative to the output's size
    assert maxabs(Y, Yr) <= 1e-4 * max(1.0, Yr.abs().max().item()), (maxabs(Y, Yr), Yr.abs().max().item())
    assert maxabs(st[:, :, :D - r, :D], Sr) <= 1e-4


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("T", [1, 100, 257])
def test_outlier_attention(dtype, T):
    from outlierneuronattention_b200 import exact_attention_triton
    B, H, D, r = 2, 3, 64, 16
    q, k, v, _, mix, _ = rand_qkv(B, H, T, D, dtype, seed=T + 1, scale=1.0)
    base = (torch.randn(B, H, T, D, generator=torch.Generator().manual_seed(T)) * 0.1).to(dtype)
    out = base.cuda().clone()
    exact_attention_triton(q.cuda(), k.cuda(), v.cuda(), r, 2.0, mix.cuda(), out=out)
    ref = outlier_attention_core(q, k, v, r, 2.0, mix, out=base)
    assert maxabs(out, ref) <= (1e-4 if dtype == torch.float32 else 2e-2)


@pytest.mark.parametrize("D,r", [(128, 32), (32, 8), (64, 32), (128, 64), (64, 12)])
def test_outlier_attention_shapes(D, r):
    from outlierneuronattention_b200 import exact_attention_triton
    B, H, T = 1, 2, 190
    q, k, v, _, mix, _ = rand_qkv(B, H, T, D, torch.bfloat16, seed=D + r, scale=1.0)
    out = exact_attention_triton(q.cuda(), k.cuda(), v.cuda(), r, math.sqrt(D / r), mix.cuda())
    ref = outlier_attention_core(q, k, v, r, math.sqrt(D / r), mix)
    assert maxabs(out, ref) <= 2e-2


def test_outlier_attention_query_suffix_with_offset():
    from outlierneuronattention_b200 import exact_attention_triton
    B, H, T, D, r = 1, 2, 300, 64, 16
    q, k, v, _, mix, _ = rand_qkv(B, H, T, D, torch.bfloat16, seed=77, scale=1.0)
    out = exact_attention_triton(q[:, :, 170:].cuda(), k.cuda(), v.cuda(), r, 2.0, mix[:, :, 170:].cuda(),
                                 q_offset=170, accumulate=False)
    ref = outlier_attention_core(q[:, :, 170:], k, v, r, 2.0, mix[:, :, 170:], q_offset=170)
    assert maxabs(out, ref) <= 2e-2


def _full_size_check(B, H, T, q, k, v, lg, mix, heads, row_blocks, label):
    """Runs the GLA and the attention on the GPU at full size (as the layer
    does: GLA writes Y, attention adds into it) and checks the sampled
    (b, h) heads against the oracle: every GLA row and the final GLA state,
    and the attention at 128-row blocks starting at ``row_blocks``.
    Returns the achieved max-abs errors (also printed)."""
    from outlierneuronattention_b200 import chunk_gla_inlier_fwd, exact_attention_triton
    D, r = 64, 16
    gs = torch.ones(1, H, 1, D, device="cuda")
    Y, st = chunk_gla_inlier_fwd(q, k, v, lg, r, 64, mix_g=mix, gla_scale=gs)
    Y_gla = Y.clone()
    exact_attention_triton(q, k, v, r, 2.0, mix, out=Y)
    torch.cuda.synchronize()
    assert torch.isfinite(Y.float()).all()
    assert _prefill_status() == 0
    e_gla = e_state = e_attn = 0.0
    smax = 0.0
    for (b, h) in heads:
        sl = lambda t: t[b:b + 1, h:h + 1].cpu()
        Yr, Sr = chunk_gla_core(sl(q), sl(k), sl(v), sl(lg), r, 64, mix_g=sl(mix), gla_scale=gs[:, h:h + 1].cpu(),
                                eps=1e-5)
        e_gla = max(e_gla, maxabs(sl(Y_gla), Yr))
        e_state = max(e_state, maxabs(sl(st)[:, :, :D - r, :D], Sr))
        smax = max(smax, Sr.abs().max().item())
        for q0 in row_blocks:
            ref = outlier_attention_core(sl(q)[:, :, q0:q0 + 128], sl(k), sl(v), r, 2.0, sl(mix)[:, :, q0:q0 + 128],
                                         out=sl(Y_gla)[:, :, q0:q0 + 128], q_offset=q0)
            e_attn = max(e_attn, maxabs(sl(Y)[:, :, q0:q0 + 128], ref))
    print(f"{label}: max-abs GLA output {e_gla:.3e}, GLA state {e_state:.3e} (|S| max {smax:.2f}), "
          f"attention output {e_attn:.3e} over {len(heads)} heads x {len(row_blocks) * 128} attention rows")
    assert e_gla <= 2e-2 and e_state <= 2e-2 and e_attn <= 2e-2, (e_gla, e_state, e_attn)
    return e_gla, e_state, e_attn


def test_config2_full_size_sampled_heads():
    """BASELINE config 2 (B=4, T=8192, H=16, d_h=64, r=16) in bf16 on the GPU;
    eight (b, h) heads spread over the batch are checked against the oracle:
    every GLA row, the final GLA state, and 16 attention blocks of 128 query
    rows spread evenly over the sequence (2,048 rows per head, first and last
    block included)."""
    B, H, T = 4, 16, 8192
    g = torch.Generator(device="cuda").manual_seed(2)
    q = torch.randn(B, H, T, 64, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, H, T, 64, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, H, T, 64, device="cuda", generator=g).to(torch.bfloat16)
    lg = F.logsigmoid(torch.randn(B, H, T, device="cuda", generator=g) + 2.0)
    mix = torch.sigmoid(torch.randn(B, H, T, device="cuda", generator=g)).to(torch.bfloat16)
    heads = [(0, 0), (0, 9), (1, 3), (1, 14), (2, 6), (2, 11), (3, 1), (3, 15)]
    rows = [i * (T - 128) // 15 // 128 * 128 for i in range(16)]
    assert rows[0] == 0 and rows[-1] == T - 128
    _full_size_check(B, H, T, q, k, v, lg, mix, heads, rows, "config 2")


def test_config4_full_size_sampled_heads():
    """BASELINE config 4 (B=1, T=65536, H=16, d_h=64, r=16) in bf16 on the GPU:
    the attention kernel's 1,024-tile key loop and the GLA's 512-chunk scan at
    full length.  Four heads against the oracle: every GLA row and the final
    state, and attention blocks at the start, the middle and the end.  Heads
    8-15 get keys whose outlier channel 0 grows along the sequence (logits rise
    by about 150 log2 units from the first key to the last), so the running
    max of late rows is raised far beyond the lazy-rescale threshold many
    times deep into the key loop; heads 0-7 are N(0, 1)."""
    B, H, T = 1, 16, 65536
    g = torch.Generator(device="cuda").manual_seed(4)
    q = torch.randn(B, H, T, 64, device="cuda", generator=g)
    k = torch.randn(B, H, T, 64, device="cuda", generator=g)
    v = torch.randn(B, H, T, 64, device="cuda", generator=g)
    q[:, 8:, :, 0] = 1.0 + 0.1 * q[:, 8:, :, 0]
    k[:, 8:, :, 0] = 0.8 * k[:, 8:, :, 0] + 52.0 * torch.arange(T, device="cuda") / T
    q, k, v = (t.to(torch.bfloat16) for t in (q, k, v))
    lg = F.logsigmoid(torch.randn(B, H, T, device="cuda", generator=g) + 2.0)
    mix = torch.sigmoid(torch.randn(B, H, T, device="cuda", generator=g)).to(torch.bfloat16)
    heads = [(0, 2), (0, 7), (0, 8), (0, 13)]
    rows = [0, 128, 8192, 32768 - 128, 32768, 49152, T - 256, T - 128]
    _full_size_check(B, H, T, q, k, v, lg, mix, heads, rows, "config 4")


def _prefill_status():
    import ctypes
    from outlierneuronattention_b200 import _capi
    v = ctypes.c_int32(0)
    assert _capi.lib().hofa_prefill_read_status(_capi.stream_handle(torch.device("cuda")), ctypes.byref(v)) == 0
    return v.value


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,H,T,D,r,qoff", [(1, 1, 128, 64, 16, 0), (2, 3, 1000, 64, 16, 0), (1, 2, 129, 64, 16, 0),
                                            (1, 2, 300, 128, 32, 0), (1, 2, 256, 64, 64, 0), (1, 2, 200, 64, 16, 77),
                                            (2, 2, 257, 128, 16, 0)])
def test_outlier_tensor_core_path(monkeypatch, dtype, B, H, T, D, r, qoff):
    """The tcgen05 kernel (bf16/f16, D in {64,128}, r in {16,32,64}) and the
    CUDA-core kernel agree with the oracle on the same inputs; the tensor-core
    kernel's bounded waits never ran out."""
    from outlierneuronattention_b200 import exact_attention_triton
    q, k, v, _, mix, _ = rand_qkv(B, H, T, D, dtype, seed=T + D + r, scale=1.0)
    qs, ms = q[:, :, qoff:], mix[:, :, qoff:]
    base = (torch.randn(B, H, T - qoff, D, generator=torch.Generator().manual_seed(T + D)) * 0.1).to(dtype)
    ref = outlier_attention_core(qs, k, v, r, math.sqrt(D / r), ms, out=base, q_offset=qoff)
    assert _prefill_status() == 0
    outs = {}
    for path in ("tc", "cuda_core"):
        if path == "cuda_core":
            monkeypatch.setenv("HOFA_OUTLIER_NO_TC", "1")
        out = base.cuda().clone()
        exact_attention_triton(qs.cuda(), k.cuda(), v.cuda(), r, math.sqrt(D / r), ms.cuda(), out=out, q_offset=qoff)
        torch.cuda.synchronize()
        outs[path] = out
        assert maxabs(out, ref) <= 2e-2, path
    monkeypatch.delenv("HOFA_OUTLIER_NO_TC")
    assert _prefill_status() == 0
    assert maxabs(outs["tc"], outs["cuda_core"].cpu()) <= 2e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,H,T,r,fuse,init,D", [(1, 1, 128, 16, True, False, 64), (2, 3, 1000, 16, True, True, 64),
                                                 (1, 2, 129, 16, False, False, 64), (1, 2, 300, 0, True, False, 64),
                                                 (2, 2, 257, 32, True, True, 64), (1, 1, 64, 8, False, True, 64),
                                                 (1, 1, 128, 16, True, False, 128), (2, 2, 300, 32, True, True, 128),
                                                 (1, 2, 257, 64, False, False, 128), (2, 1, 129, 8, True, True, 128),
                                                 (1, 1, 200, 0, True, False, 128), (1, 1, 1000, 16, True, True, 128)])
def test_gla_tensor_core_path(monkeypatch, dtype, B, H, T, r, fuse, init, D):
    """The chunk-parallel tcgen05 GLA (bf16/f16, d_h = 64 or 128, scalar decay)
    and the CUDA-core GLA agree with the oracle on the same inputs, including a
    seeded initial state; the tensor-core kernels' bounded waits never ran out."""
    from outlierneuronattention_b200.chunk_gla_inlier import gla_forward
    q, k, v, lg, mix, gs = rand_qkv(B, H, T, D, dtype, seed=T + r, scale=0.3)
    s0 = torch.randn(B, H, D - r, D, generator=torch.Generator().manual_seed(T + r)) * 0.3 if init else None
    Yr, Sr = chunk_gla_core(q, k, v, lg, r, 64, mix_g=mix if fuse else None, gla_scale=gs if fuse else None,
                            eps=1e-5, state_init=s0)
    assert fuse or Yr.abs().max().item() < 4.0  # raw outputs: the bf16 output's own rounding stays below 1e-2
    assert _prefill_status() == 0
    outs = {}
    for path in ("tc", "cuda_core"):
        if path == "cuda_core":
            monkeypatch.setenv("HOFA_GLA_NO_TC", "1")
        st = torch.empty(B, H, D - r, D, device="cuda")
        Y = gla_forward(q.cuda(), k.cuda(), v.cuda(), lg.cuda(), r, mix_g=mix.cuda() if fuse else None,
                        gla_scale=gs.cuda() if fuse else None, state_out=st,
                        initial_state=None if s0 is None else s0.cuda())
        torch.cuda.synchronize()
        outs[path] = (Y, st)
        assert maxabs(Y, Yr) <= 2e-2, path
        assert maxabs(st, Sr) <= 2e-2, path
    monkeypatch.delenv("HOFA_GLA_NO_TC")
    assert _prefill_status() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,H,T,r,D,decay,fuse", [(1, 2, 300, 16, 64, "weak", True), (2, 2, 257, 32, 64, "mixed", True),
                                                  (1, 2, 1000, 16, 64, "strong", True), (1, 1, 200, 8, 64, "mixed", False),
                                                  (2, 1, 300, 32, 128, "weak", True), (1, 2, 640, 16, 128, "mixed", True),
                                                  (1, 1, 500, 64, 128, "strong", False)])
def test_gla_tensor_core_per_channel_decay(monkeypatch, dtype, B, H, T, r, D, decay, fuse):
    """learnable_alpha on the tensor cores (the reference's factored decay,
    src/chunk_gla_inlier.py:90-107, over key sub-blocks of 64, 32 or 16 tokens
    chosen per chunk so that the factors stay in range, exact CUDA-core scores
    beyond that; the decayed operands as hi + lo 16-bit terms) and the CUDA-core
    kernel agree with the float64 oracle, output and final state, with a seeded
    initial state; every output is finite (the reference's own form, with its
    single rounding at 64-token chunks, overflows to NaN on the mixed and strong
    inputs: ``chunk_gla_reference_rounding``); no bounded wait ran out."""
    from outlierneuronattention_b200.chunk_gla_inlier import gla_forward
    q, k, v, lg, mix, gs = rand_qkv(B, H, T, D, dtype, seed=T + r + D, scale=0.3)
    g = torch.Generator().manual_seed(T * 7 + D)
    mu = {"weak": 4.0, "mixed": 1.0, "strong": -1.0}[decay]
    lg = F.logsigmoid(torch.randn(B, H, T, generator=g) * (1.0 if decay != "mixed" else 2.0) + mu)
    la = torch.randn(1, H, 1, D - r, generator=g) * 0.5
    s0 = torch.randn(B, H, D - r, D, generator=g) * 0.3
    kw = dict(log_alpha=la, mix_g=mix if fuse else None, gla_scale=gs if fuse else None, eps=1e-5, state_init=s0)
    Yr, Sr = chunk_gla_core(q, k, v, lg, r, 64, **kw)
    assert fuse or Yr.abs().max().item() < 4.0  # raw outputs: the 16-bit output's own rounding stays below 1e-2
    assert _prefill_status() == 0
    for path in ("tc", "cuda_core"):
        if path == "cuda_core":
            monkeypatch.setenv("HOFA_GLA_NO_TC", "1")
        st = torch.empty(B, H, D - r, D, device="cuda")
        Y = gla_forward(q.cuda(), k.cuda(), v.cuda(), lg.cuda(), r, log_alpha=la.cuda(),
                        mix_g=mix.cuda() if fuse else None, gla_scale=gs.cuda() if fuse else None,
                        state_out=st, initial_state=s0.cuda())
        torch.cuda.synchronize()
        assert torch.isfinite(Y).all(), path
        assert maxabs(Y, Yr) <= 2e-2, (path, maxabs(Y, Yr))
        assert maxabs(st, Sr) <= 2e-2, (path, maxabs(st, Sr))
    monkeypatch.delenv("HOFA_GLA_NO_TC")
    assert _prefill_status() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_outlier_tensor_core_growing_logits(dtype):
    """Scores that grow along the keys (about 0.7 log2 units per key, 90 over
    128 keys): later tiles raise the running max far past the lazy-rescale
    threshold, so rows of O are rescaled in TMEM mid-sequence."""
    from outlierneuronattention_b200.exact_attention import exact_attention_triton
    B, H, T, D, r = 1, 2, 320, 64, 16
    g = torch.Generator().manual_seed(77)
    q = torch.zeros(B, H, T, D)
    q[..., :r] = 1.0 + 0.05 * torch.randn(B, H, T, r, generator=g)
    k = torch.zeros(B, H, T, D)
    k[..., :r] = (torch.arange(T, dtype=torch.float32) / 64).view(1, 1, T, 1) * (1 + 0.05 * torch.randn(B, H, T, r, generator=g))
    v = torch.randn(B, H, T, D, generator=g)
    mix = torch.sigmoid(torch.randn(B, H, T, generator=g))
    q, k, v, mix = (t.to(dtype) for t in (q, k, v, mix))
    out = exact_attention_triton(q.cuda(), k.cuda(), v.cuda(), r, 2.0, mix.cuda(),
                                 out=torch.zeros(B, H, T, D, dtype=dtype, device="cuda"))
    torch.cuda.synchronize()
    ref = outlier_attention_core(q, k, v, r, 2.0, mix)
    assert torch.isfinite(out.float()).all()
    assert maxabs(out, ref) <= 2e-2
    assert _prefill_status() == 0
