"""The decoder LM harness and its graph-replayed decode engine.

* the engine (device-side position, sampling inside a CUDA graph of two decode
  steps) produces exactly what an eager loop over the same ``HofaLM.step``
  produces from the same prefill (the same greedy tokens);
* the fused small-batch step (``hofa_lm_linear_fwd`` projections with RMSNorm,
  SwiGLU and the residual folded in, around the layer's one-launch decode
  step) matches the modules run as written (the layer's ``forward_step``,
  nn.RMSNorm, nn.Linear) within bf16 rounding;
* ``hofa_lm_linear_fwd`` matches a float32 PyTorch computation of each input
  mode.
"""
import pytest
import torch
import torch.nn.functional as F

from outlierneuronattention_b200.lm import DecodeEngine, HofaLM, LMConfig, lm_linear, sample_tokens

pytestmark = pytest.mark.gpu


def _model(dtype, vocab=1000, d_model=256, heads=4, layers=2, mlp=512):
    torch.manual_seed(0)
    cfg = LMConfig(vocab_size=vocab, d_model=d_model, num_heads=heads, num_layers=layers, r=16, d_mlp=mlp)
    return HofaLM(cfg).to(device="cuda", dtype=dtype).eval(), cfg


@pytest.mark.parametrize("dtype,B", [(torch.float32, 3), (torch.bfloat16, 3), (torch.bfloat16, 12)])
def test_engine_matches_eager_loop(dtype, B):
    m, cfg = _model(dtype)
    T, n = 96, 10
    prompt = torch.randint(0, cfg.vocab_size, (B, T), generator=torch.Generator().manual_seed(1)).cuda()
    with torch.no_grad():
        logits0, caches, states = m.prefill(prompt, capacity=T + n + 2)
        eng = DecodeEngine(m, caches, states, logits0, T)
        eng.capture(n)
        toks = eng.generate(n)
        toks_again = eng.generate(n)   # every call starts again from the prompt
        torch.cuda.synchronize()
        # eager loop over the same step function, from a fresh prefill
        logits0b, caches_b, states_b = m.prefill(prompt, capacity=T + n + 2)
        tok = logits0b.argmax(-1)[:, None]
        ref = [tok]
        for i in range(n):
            pos = torch.tensor([T + i], dtype=torch.int32, device="cuda")
            tok = m.step(tok, caches_b, states_b, pos, flip=i % 2 == 1).argmax(-1)[:, None]
            ref.append(tok)
        ref = torch.cat(ref, 1)
    assert toks.shape == (B, n + 1)
    assert torch.equal(toks, ref)
    assert torch.equal(toks, toks_again)
    eng.release()


@pytest.mark.parametrize("B", [1, 4, 8])
def test_fused_step_matches_modules(B):
    m, cfg = _model(torch.bfloat16, vocab=2000, d_model=512, heads=8, layers=2, mlp=1024)
    T = 80
    prompt = torch.randint(0, cfg.vocab_size, (B, T), generator=torch.Generator().manual_seed(2)).cuda()
    tok = torch.randint(0, cfg.vocab_size, (B, 1), generator=torch.Generator().manual_seed(3)).cuda()
    pos = torch.tensor([T], dtype=torch.int32, device="cuda")
    outs = {}
    with torch.no_grad():
        for fused in (True, False):
            _, caches, states = m.prefill(prompt, capacity=T + 4)
            outs[fused] = (m.step(tok, caches, states, pos, flip=False, fused=fused).float(),
                           [s[1].clone() for s in states], [c[0][:, :, T].clone() for c in caches])
    lf, lu = outs[True][0], outs[False][0]
    scale = lu.abs().max().item()
    assert (lf - lu).abs().max().item() <= 3e-2 * max(1.0, scale), ((lf - lu).abs().max().item(), scale)
    for a, b in zip(outs[True][1], outs[False][1]):       # GLA states after the step
        assert (a - b).abs().max().item() <= 2e-2
    for a, b in zip(outs[True][2], outs[False][2]):       # the appended cache row
        assert (a.float() - b.float()).abs().max().item() <= 2e-2


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("M,N,K", [(1, 3072, 1024), (4, 1000, 4096), (8, 264, 2048), (3, 32000, 1024),
                                   (1, 9001, 1024), (1, 1024, 4096), (1, 520, 2048)])
def test_lm_linear_modes(mode, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + mode)
    x = torch.randn(M, 2 * K if mode == 2 else K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.03).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(K, device="cuda", generator=g)).to(torch.bfloat16)
    res = torch.randn(M, N, device="cuda", generator=g).to(torch.bfloat16)
    y = res.clone()
    lm_linear(x, w, y, norm_w=nw if mode == 1 else None, residual=y, mode=mode, eps=1e-6)
    xf = x.float()
    if mode == 1:
        xin = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * nw.float()).to(torch.bfloat16).float()
    elif mode == 2:
        xin = (F.silu(xf[:, :K]).to(torch.bfloat16).float() * xf[:, K:]).to(torch.bfloat16).float()
    else:
        xin = xf
    ref = res.float() + xin @ w.float().t()
    assert (y.float() - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item())


def test_sampling_on_device_is_a_top_k_draw():
    torch.manual_seed(3)
    logits = torch.randn(4, 1000, device="cuda")
    top = logits.topk(5, dim=-1).indices
    for _ in range(20):
        t = sample_tokens(logits, 1.0, 5)
        assert t.shape == (4,)
        assert (t[:, None] == top).any(-1).all()
    assert torch.equal(sample_tokens(logits, 0.0, 5), logits.argmax(-1))
