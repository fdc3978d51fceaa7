"""The decoder LM harness and its graph-replayed decode engine.

The engine (device-side position, sampling inside a CUDA graph of two decode
steps) must produce what an eager host loop over the same model produces:
the same greedy tokens and the same logits, starting from the same prefill.
The eager loop passes the position as a host integer (the layer's other
pre-allocated-cache path), so both positions paths of the layer are compared.
"""
import pytest
import torch

from outlierneuronattention_b200.lm import DecodeEngine, HofaLM, LMConfig, sample_tokens

pytestmark = pytest.mark.gpu


def _model(dtype):
    torch.manual_seed(0)
    cfg = LMConfig(vocab_size=1000, d_model=256, num_heads=4, num_layers=2, r=16, d_mlp=512)
    return HofaLM(cfg).to(device="cuda", dtype=dtype).eval(), cfg


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_engine_matches_eager_greedy_loop(dtype):
    m, cfg = _model(dtype)
    B, T, n = 3, 96, 10
    prompt = torch.randint(0, cfg.vocab_size, (B, T), generator=torch.Generator().manual_seed(1)).cuda()
    with torch.no_grad():
        logits0, caches, states = m.prefill(prompt, capacity=T + n + 2)
        eng = DecodeEngine(m, caches, states, logits0, T)
        eng.capture(n)
        toks = eng.generate(n)
        toks_again = eng.generate(n)   # every call starts again from the prompt
        torch.cuda.synchronize()
        # eager loop with host positions, from a fresh prefill
        logits0b, caches_b, states_b = m.prefill(prompt, capacity=T + n + 2)
        tok = logits0b.argmax(-1)[:, None]
        ref = [tok]
        st = [(s0, s1) for s0, s1 in states_b]
        for i in range(n):
            x = m.embed(tok)
            for blk, cache, j in zip(m.blocks, caches_b, range(len(st))):
                y, _, st[j] = blk.attn.forward_step(blk.attn_norm(x), cache, st[j], cache_seq_len=T + i)
                x = x + y
                x = x + blk.mlp(blk.mlp_norm(x))
            logits = m.logits(x[:, -1])
            tok = logits.argmax(-1)[:, None]
            ref.append(tok)
        ref = torch.cat(ref, 1)
    assert toks.shape == (B, n + 1)
    assert torch.equal(toks, ref)
    assert torch.equal(toks, toks_again)
    eng.release()


def test_sampling_on_device_is_a_top_k_draw():
    torch.manual_seed(3)
    logits = torch.randn(4, 1000, device="cuda")
    top = logits.topk(5, dim=-1).indices
    for _ in range(20):
        t = sample_tokens(logits, 1.0, 5)
        assert t.shape == (4,)
        assert (t[:, None] == top).any(-1).all()
    assert torch.equal(sample_tokens(logits, 0.0, 5), logits.argmax(-1))
