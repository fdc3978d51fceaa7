"""hofa_decode_step_fwd: the decode step with the new token's prep in the same launch.

The fused step must give what the two launches give (hofa_prep_fwd, then
hofa_decode_fwd over the appended cache): the output Y, the new GLA state, the
appended cache row, log_gamma and mix.  The two-launch form runs on copies of
the inputs (it rotates q and k in place).  The layer-level decode tests
(test_module_gpu.py) cover the fused step against the oracle, because the
layer's pre-allocated-cache path uses it.
"""
import pytest
import torch
import torch.nn.functional as F

from outlierneuronattention_b200 import fused_hofa_decode
from outlierneuronattention_b200.hofa_decode import fused_hofa_decode_step
from outlierneuronattention_b200.modules import RotaryEmbedding
from outlierneuronattention_b200.prep import prep

pytestmark = pytest.mark.gpu


def _case(B, H, D, R, L, dtype, seed, fixed_mix=False, alpha=False, rope=True):
    g = torch.Generator().manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=g)
    dev = "cuda"
    c = dict(q=rn(B, H, 1, D).to(dtype).to(dev), k=rn(B, H, 1, D).to(dtype).to(dev), v=rn(B, H, 1, D).to(dtype).to(dev),
             cache_k=(2 * rn(B, H, L, R)).to(dtype).to(dev), cache_v=(0.6 * rn(B, H, L, D)).to(dtype).to(dev),
             state=(0.1 * rn(B, H, D - R, D)).to(dev), norm_w=(1 + 0.2 * rn(H, D)).to(dev),
             gate_w=(0.1 * rn(H, 2 * D)).to(dev), gate_b=torch.full((H,), -1.0, device=dev))
    if fixed_mix:
        c["fixed_mix"] = rn(H).to(dev)
    else:
        c["mix_w"], c["mix_b"] = (0.1 * rn(H, 2 * D)).to(dev), (0.1 * rn(H)).to(dev)
    if alpha:
        c["log_alpha"] = (0.3 * rn(1, H, 1, D - R)).to(dev)
    if rope:
        re = RotaryEmbedding(R).to(dev)
        re(L + 1)
        c["cos"], c["sin"] = re.cos_cached, re.sin_cached
    return c


def _two_launches(c, R, seq_len, split_k):
    q, k = c["q"].clone(), c["k"].clone()
    ck, cv = c["cache_k"].clone(), c["cache_v"].clone()
    B, H = q.shape[:2]
    lg = torch.empty(B, H, 1, device="cuda")
    mix = torch.empty(B, H, 1, device="cuda", dtype=q.dtype)
    gk = {n: c[n] for n in ("mix_w", "mix_b", "fixed_mix") if n in c}
    prep(q, k, c["v"], c["gate_w"], c["gate_b"], lg, mix_out=mix, cos=c.get("cos"), sin=c.get("sin"), R=R,
         pos0=seq_len - 1, cache_k=ck, cache_v=cv, use_rope="cos" in c, **gk)
    st = torch.empty_like(c["state"])
    y = fused_hofa_decode(q, k, c["v"], ck, cv, c["state"], st, lg, mix, c["norm_w"], R, seq_len, 2.0,
                          split_k=split_k, log_alpha=c.get("log_alpha"))
    return y, st, ck, cv, lg, mix


def _fused(c, R, seq_len, split_k, seq_len_dev=None):
    ck, cv = c["cache_k"].clone(), c["cache_v"].clone()
    st = torch.empty_like(c["state"])
    gk = {n: c[n] for n in ("mix_w", "mix_b", "fixed_mix") if n in c}
    y, lg, mix = fused_hofa_decode_step(c["q"].clone(), c["k"].clone(), c["v"], ck, cv, c["state"], st, c["norm_w"], R,
                                        seq_len, 2.0, c["gate_w"], c["gate_b"], cos=c.get("cos"), sin=c.get("sin"),
                                        log_alpha=c.get("log_alpha"), split_k=split_k, seq_len_dev=seq_len_dev, **gk)
    return y, st, ck, cv, lg, mix


def _compare(a, b, tol=2e-2):
    ya, sa, cka, cva, lga, mxa = a
    yb, sb, ckb, cvb, lgb, mxb = b
    torch.cuda.synchronize()
    assert torch.isfinite(ya.float()).all()
    assert (ya.float() - yb.float()).abs().max().item() <= tol
    torch.testing.assert_close(sa, sb, atol=1e-5, rtol=1e-5)
    assert torch.equal(cka, ckb) and torch.equal(cva, cvb)
    torch.testing.assert_close(lga, lgb, atol=1e-6, rtol=1e-6)
    assert torch.equal(mxa, mxb)


@pytest.mark.parametrize("B,H,D,R,L,seq_len,dtype,split", [
    (4, 16, 64, 16, 4096, 4096, torch.bfloat16, None),
    (1, 16, 64, 16, 4096, 4096, torch.bfloat16, None),
    (2, 4, 64, 16, 1500, 1000, torch.bfloat16, 4),
    (2, 4, 64, 16, 1500, 1000, torch.bfloat16, 24),
    (2, 4, 64, 16, 300, 1, torch.bfloat16, None),      # first token: empty cache before it
    (2, 4, 64, 16, 300, 2, torch.bfloat16, 1),
    (2, 4, 64, 16, 300, 65, torch.float16, None),
    (2, 4, 128, 32, 700, 700, torch.bfloat16, None),
    (3, 2, 128, 64, 200, 130, torch.bfloat16, 2),
])
def test_fused_step_matches_two_launches(B, H, D, R, L, seq_len, dtype, split):
    c = _case(B, H, D, R, L, dtype, seed=seq_len + R)
    _compare(_fused(c, R, seq_len, split), _two_launches(c, R, seq_len, split))


@pytest.mark.parametrize("variant", ["fixed_mix", "alpha", "no_rope"])
def test_fused_step_variants(variant):
    c = _case(2, 4, 64, 16, 800, torch.bfloat16, seed=7, fixed_mix=variant == "fixed_mix",
              alpha=variant == "alpha", rope=variant != "no_rope")
    _compare(_fused(c, 16, 777, None), _two_launches(c, 16, 777, None))


def test_fused_step_device_seq_len_in_cuda_graph():
    """Position from a device int32 (seq_len - 1) under CUDA-graph replay."""
    c = _case(2, 4, 64, 16, 600, torch.bfloat16, seed=11)
    sl = torch.tensor([300], dtype=torch.int32, device="cuda")
    ck, cv = c["cache_k"].clone(), c["cache_v"].clone()
    st = torch.empty_like(c["state"])
    q, k = c["q"].clone(), c["k"].clone()
    gk = dict(mix_w=c["mix_w"], mix_b=c["mix_b"])
    args = (q, k, c["v"], ck, cv, c["state"], st, c["norm_w"], 16, 600, 2.0, c["gate_w"], c["gate_b"])
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        fused_hofa_decode_step(*args, cos=c["cos"], sin=c["sin"], seq_len_dev=sl, **gk)  # warm-up
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            out = fused_hofa_decode_step(*args, cos=c["cos"], sin=c["sin"], seq_len_dev=sl, **gk)
        for n in (300, 451):
            sl.fill_(n)
            ck.copy_(c["cache_k"])
            cv.copy_(c["cache_v"])
            g.replay()
            s.synchronize()
            ref = _two_launches(c, 16, n, None)
            _compare((out[0], st, ck, cv, out[1], out[2]), ref)
    del g


def test_fused_step_rejects_mismatched_tensors():
    from outlierneuronattention_b200._capi import HofaError
    c = _case(1, 2, 64, 16, 64, torch.bfloat16, seed=3)
    st = torch.empty_like(c["state"])
    with pytest.raises(HofaError):
        fused_hofa_decode_step(c["q"], c["k"], c["v"], c["cache_k"], c["cache_v"], c["state"], st, c["norm_w"], 16,
                               65, 2.0, c["gate_w"], c["gate_b"], mix_w=c["mix_w"], mix_b=c["mix_b"])  # seq_len > L
