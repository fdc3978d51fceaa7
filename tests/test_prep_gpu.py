"""hofa_prep_fwd (gates, logsigmoid, RoPE in place, cache rows) against the
reference's formulas (src/HybridOutlierFactorizedAttention.py:67-95, 176-198,
365-384; src/modules/modules.py:33-45) evaluated in float64 on the same inputs.
Both kernels are covered: the 16-byte-row kernel (bf16 views of a
projection output) and the warp-per-token kernel (strided / float32)."""
import pytest
import torch
import torch.nn.functional as F

from oracle.hofa_oracle import apply_rope, rope_cos_sin

pytestmark = pytest.mark.gpu


def reference(q, k, v, gw, gb, mw, mb, r, pos0, base=10000.0):
    q, k, v = q.double(), k.double(), v.double()
    D = q.shape[-1]
    logits = torch.einsum("bhnf,hf->bhn", q, gw[:, :D].double()) + torch.einsum("bhnf,hf->bhn", k, gw[:, D:].double()) + gb.double().view(1, -1, 1)
    ml = torch.einsum("bhnf,hf->bhn", q, mw[:, :D].double()) + torch.einsum("bhnf,hf->bhn", k, mw[:, D:].double()) + mb.double().view(1, -1, 1)
    N = q.shape[2]
    cos, sin = rope_cos_sin(r, pos0 + N, base)
    cos, sin = cos[pos0:], sin[pos0:]
    qr, kr = q.clone(), k.clone()
    if r:
        qr[..., :r] = apply_rope(q[..., :r], cos, sin)
        kr[..., :r] = apply_rope(k[..., :r], cos, sin)
    return F.logsigmoid(-logits), torch.sigmoid(ml), qr, kr


@pytest.mark.parametrize("dtype,strided", [(torch.bfloat16, False), (torch.float16, False), (torch.float32, False),
                                           (torch.bfloat16, True)])
@pytest.mark.parametrize("D,r", [(64, 16), (64, 32), (128, 32), (64, 0)])
def test_prep_matches_reference_formulas(dtype, strided, D, r):
    from outlierneuronattention_b200.modules import RotaryEmbedding
    from outlierneuronattention_b200.prep import prep
    g = torch.Generator().manual_seed(D + r)
    B, H, N, L, pos0 = 2, 3, 150, 300, 17
    x = torch.randn(B, N, 3, H, D, generator=g)
    if strided:  # channel stride 2: the warp-per-token kernel
        x = torch.randn(B, N, 3, H, D, 2, generator=g)[..., 0]
    xq, xk, xv = (x[:, :, i].transpose(1, 2) for i in range(3))  # [B,H,N,D] views
    gw, mw = torch.randn(H, 2 * D, generator=g) * 0.3, torch.randn(H, 2 * D, generator=g) * 0.3
    gb, mb = torch.randn(H, generator=g), torch.randn(H, generator=g)
    qd, kd, vd = (t.to(dtype).cuda() for t in (xq, xk, xv))
    ref_lg, ref_mix, ref_q, ref_k = reference(qd.cpu(), kd.cpu(), vd.cpu(), gw, gb, mw, mb, r, pos0)
    lg = torch.empty(B, H, N, device="cuda")
    mix = torch.empty(B, H, N, device="cuda", dtype=dtype)
    ck = torch.zeros(B, H, L, max(r, 8), device="cuda", dtype=dtype)
    cv = torch.zeros(B, H, L, D, device="cuda", dtype=dtype)
    rope = RotaryEmbedding(max(r, 2)).cuda()
    prep(qd, kd, vd, gw.cuda(), gb.cuda(), lg, mix_w=mw.cuda(), mix_b=mb.cuda(), mix_out=mix,
         cos=rope.cos_cached, sin=rope.sin_cached, R=r, pos0=pos0, cache_k=ck if r else None, cache_v=cv,
         use_rope=r > 0)
    torch.cuda.synchronize()
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    assert (lg.double().cpu() - ref_lg).abs().max().item() <= tol
    assert (mix.double().cpu() - ref_mix).abs().max().item() <= tol
    assert (qd.double().cpu() - ref_q).abs().max().item() <= tol * 4
    assert (kd.double().cpu() - ref_k).abs().max().item() <= tol * 4
    if r:
        assert (ck[:, :, pos0:pos0 + N, :r].double().cpu() - ref_k[..., :r]).abs().max().item() <= tol * 4
        assert ck[:, :, :pos0].abs().max().item() == 0 and ck[:, :, pos0 + N:].abs().max().item() == 0
    assert torch.equal(cv[:, :, pos0:pos0 + N].cpu(), vd.cpu())


@pytest.mark.parametrize("layout", ["token_major", "head_major"])
@pytest.mark.parametrize("D,r", [(32, 8), (32, 32), (64, 8), (64, 16), (64, 64), (128, 16), (128, 64)])
def test_prep_row_layouts(layout, D, r):
    """Both 16-byte-row kernels: token_major views of one [B, N, 3, H, D]
    projection output (a token's heads adjacent: the warp-per-token kernel)
    and head_major separate [B, H, N, D] tensors (the thread-per-row kernel).
    H = 5 leaves part of a warp's 16-byte slots without a head."""
    from outlierneuronattention_b200.modules import RotaryEmbedding
    from outlierneuronattention_b200.prep import prep
    dtype = torch.bfloat16
    g = torch.Generator().manual_seed(7 * D + r)
    B, H, N, L, pos0 = 2, 5, 70, 100, 9
    x = torch.randn(B, N, 3, H, D, generator=g).to(dtype)
    if layout == "token_major":
        xd = x.cuda()
        qd, kd, vd = (xd[:, :, i].transpose(1, 2) for i in range(3))
        assert qd.stride(1) == D
    else:
        qd, kd, vd = (x[:, :, i].transpose(1, 2).contiguous().cuda() for i in range(3))
        assert qd.stride(1) == N * D
    gw, mw = torch.randn(H, 2 * D, generator=g) * 0.3, torch.randn(H, 2 * D, generator=g) * 0.3
    gb, mb = torch.randn(H, generator=g), torch.randn(H, generator=g)
    ref_lg, ref_mix, ref_q, ref_k = reference(qd.cpu(), kd.cpu(), vd.cpu(), gw, gb, mw, mb, r, pos0)
    lg = torch.empty(B, H, N, device="cuda")
    mix = torch.empty(B, H, N, device="cuda", dtype=dtype)
    ck = torch.zeros(B, H, L, r, device="cuda", dtype=dtype)
    cv = torch.zeros(B, H, L, D, device="cuda", dtype=dtype)
    rope = RotaryEmbedding(r).cuda()
    prep(qd, kd, vd, gw.cuda(), gb.cuda(), lg, mix_w=mw.cuda(), mix_b=mb.cuda(), mix_out=mix,
         cos=rope.cos_cached, sin=rope.sin_cached, R=r, pos0=pos0, cache_k=ck, cache_v=cv, use_rope=True)
    torch.cuda.synchronize()
    tol = 2e-2
    assert (lg.double().cpu() - ref_lg).abs().max().item() <= tol
    assert (mix.double().cpu() - ref_mix).abs().max().item() <= tol
    assert (qd.double().cpu() - ref_q).abs().max().item() <= tol * 4
    assert (kd.double().cpu() - ref_k).abs().max().item() <= tol * 4
    assert (ck[:, :, pos0:pos0 + N].double().cpu() - ref_k[..., :r]).abs().max().item() <= tol * 4
    assert ck[:, :, :pos0].abs().max().item() == 0 and ck[:, :, pos0 + N:].abs().max().item() == 0
    assert torch.equal(cv[:, :, pos0:pos0 + N].cpu(), vd.cpu())


@pytest.mark.parametrize("table", ["f32", "bf16", "strided"])
def test_prep_token_major_many_tokens(table):
    """More tokens than the token-major kernel has resident warps, so each warp
    walks several tokens with its (b, n) carried across batch boundaries (N is
    not a multiple of the warp count), and the RoPE tables either copied into
    the shared-memory stage with the token (contiguous float32) or read
    directly (bfloat16; float32 with channel stride 2)."""
    from outlierneuronattention_b200.modules import RotaryEmbedding
    from outlierneuronattention_b200.prep import prep
    dtype = torch.bfloat16
    g = torch.Generator().manual_seed(11)
    B, H, D, r, N, pos0 = 3, 16, 64, 16, 3001, 13
    L = N + pos0 + 7
    x = torch.randn(B, N, 3, H, D, generator=g).to(dtype)
    xd = x.cuda()
    qd, kd, vd = (xd[:, :, i].transpose(1, 2) for i in range(3))
    gw, mw = torch.randn(H, 2 * D, generator=g) * 0.3, torch.randn(H, 2 * D, generator=g) * 0.3
    gb, mb = torch.randn(H, generator=g), torch.randn(H, generator=g)
    ref_lg, ref_mix, ref_q, ref_k = reference(qd.cpu(), kd.cpu(), vd.cpu(), gw, gb, mw, mb, r, pos0)
    rope = RotaryEmbedding(r, max_seq_len=L).cuda()
    cos, sin = rope.cos_cached, rope.sin_cached
    if table == "bf16":
        cos, sin = cos.to(dtype), sin.to(dtype)
    elif table == "strided":
        wide_c = torch.zeros(cos.shape[0], 2 * r, device="cuda")
        wide_s = torch.zeros_like(wide_c)
        wide_c[:, ::2], wide_s[:, ::2] = cos, sin
        cos, sin = wide_c[:, ::2], wide_s[:, ::2]
        assert cos.stride(1) == 2
    lg = torch.empty(B, H, N, device="cuda")
    mix = torch.empty(B, H, N, device="cuda", dtype=dtype)
    ck = torch.zeros(B, H, L, r, device="cuda", dtype=dtype)
    cv = torch.zeros(B, H, L, D, device="cuda", dtype=dtype)
    prep(qd, kd, vd, gw.cuda(), gb.cuda(), lg, mix_w=mw.cuda(), mix_b=mb.cuda(), mix_out=mix,
         cos=cos, sin=sin, R=r, pos0=pos0, cache_k=ck, cache_v=cv, use_rope=True)
    torch.cuda.synchronize()
    tol = 2e-2
    assert (lg.double().cpu() - ref_lg).abs().max().item() <= tol
    assert (mix.double().cpu() - ref_mix).abs().max().item() <= tol
    assert (qd.double().cpu() - ref_q).abs().max().item() <= tol * 4
    assert (kd.double().cpu() - ref_k).abs().max().item() <= tol * 4
    assert (ck[:, :, pos0:pos0 + N].double().cpu() - ref_k[..., :r]).abs().max().item() <= tol * 4
    assert ck[:, :, :pos0].abs().max().item() == 0 and ck[:, :, pos0 + N:].abs().max().item() == 0
    assert torch.equal(cv[:, :, pos0:pos0 + N].cpu(), vd.cpu())
