"""The drop-in layer on the GPU against the reference's own outputs.

``tests/golden/*.pt`` hold per-token outputs, outlier caches and GLA states
of the reference layer (HybridOutlierFactorizedAttentionTrain.forward_step,
float64).  The drop-in ``HybridOutlierFactorizedAttention`` loads the same
state dict and must reproduce them through ``forward`` (prefill, any prefix
length) followed by ``forward_step`` (decode) in every cache mode of the
reference module (pre-allocated, concatenating, starting from no cache).

Tolerances: float32 runs <= 1e-4 max-abs; bf16 (autocast) runs <= 2e-2.
"""
import pytest
import torch

from conftest import GOLDEN_CASES, load_golden
from oracle.hofa_oracle import LayerShape, OracleLayer

pytestmark = pytest.mark.gpu


def make_layer(g, dtype=torch.float32):
    from outlierneuronattention_b200 import HybridOutlierFactorizedAttention, ModelConfig
    c = g["config"]
    cfg = ModelConfig(d_model=c["d_model"], num_heads=c["num_heads"], num_layers=1, r=c["r"],
                      chunk_size=c["chunk_size"], use_rope=c["use_rope"], rope_base=c["rope_base"],
                      learnable_alpha=c["learnable_alpha"], fixed_blend_weight=c["fixed_blend_weight"],
                      mha_heads_for_width_split=c.get("mha_heads_for_width_split", 0))
    m = HybridOutlierFactorizedAttention(cfg)
    missing, unexpected = m.load_state_dict(g["state_dict"], strict=True), None
    return m.to(device="cuda", dtype=dtype).eval()


def err(a, b):
    return (a.double().cpu() - b.double().cpu()).abs().max().item()


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_prefill_then_preallocated_decode_fp32(name):
    g = load_golden(name)
    m = make_layer(g)
    x = g["x"].cuda()
    B, T, _ = x.shape
    H, D, r = m.num_heads, m.d_head, m.r
    T0 = 50
    with torch.no_grad():
        y0, cache, state = m(x[:, :T0], return_state=True)
        assert err(y0, g["y"][:, :T0]) <= 1e-4
        assert err(state[0], g["states"][T0]) <= 1e-4
        ys = [y0]
        if r > 0:
            Kc = torch.zeros(B, H, T, r, device="cuda")
            Vc = torch.zeros(B, H, T, D, device="cuda")
            Kc[:, :, :T0] = cache[0]
            Vc[:, :, :T0] = cache[1]
            cache = (Kc, Vc)
        for t in range(T0, T):
            y, cache, state = m.forward_step(x[:, t:t + 1], cache, state, cache_seq_len=t)
            ys.append(y)
        assert err(torch.cat(ys, 1), g["y"]) <= 1e-4
        assert err(state[0], g["states"][T]) <= 1e-4
        if r > 0:
            assert err(cache[0], g["cache_k"]) <= 1e-4
            assert err(cache[1], g["cache_v"]) <= 1e-4


@pytest.mark.parametrize("name", ["mha_r_eq_dh", "width_split"])
@pytest.mark.parametrize("mode", ["preallocated", "concat", "from_empty"])
def test_ablation_branches_fp32(name, mode):
    """The reference's ablation branches against its own outputs: r == d_head
    (plain causal softmax attention, src/HybridOutlierFactorizedAttention.py:161-171,
    :333-356) and the width split (softmax heads beside GLA heads, :106-143,
    :234-296); prefill of 50 tokens then decode in each cache mode (or decode
    from no cache at all)."""
    g = load_golden(name)
    m = make_layer(g)
    x = g["x"].cuda()
    B, T, _ = x.shape
    T0 = 0 if mode == "from_empty" else 50
    cache, state, ys = None, None, []
    with torch.no_grad():
        if T0:
            y0, cache, state = m(x[:, :T0], return_state=True)
            assert err(y0, g["y"][:, :T0]) <= 1e-4
            if g["states"]:
                assert err(state[0], g["states"][T0]) <= 1e-4
            else:
                assert state is None
            ys.append(y0)
            if mode == "preallocated":
                Kc = torch.zeros(B, cache[0].shape[1], T, cache[0].shape[3], device="cuda")
                Vc = torch.zeros(B, cache[1].shape[1], T, cache[1].shape[3], device="cuda")
                Kc[:, :, :T0], Vc[:, :, :T0] = cache
                cache = (Kc, Vc)
        for t in range(T0, T):
            y, cache, state = m.forward_step(x[:, t:t + 1], cache, state,
                                             cache_seq_len=t if mode == "preallocated" else None)
            ys.append(y)
    assert err(torch.cat(ys, 1), g["y"]) <= 1e-4
    assert err(cache[0][:, :, :T], g["cache_k"]) <= 1e-4
    assert err(cache[1][:, :, :T], g["cache_v"]) <= 1e-4
    if g["states"]:
        assert err(state[0], g["states"][T]) <= 1e-4


@pytest.mark.parametrize("name", ["hofa_r16", "hofa_r16_alpha", "gla_r0"])
def test_decode_from_empty_cache_concat_mode_fp32(name):
    """forward_step from cache_O=None, then the concatenating cache mode."""
    g = load_golden(name)
    m = make_layer(g)
    x = g["x"].cuda()
    cache, state, ys = None, None, []
    with torch.no_grad():
        for t in range(x.shape[1]):
            y, cache, state = m.forward_step(x[:, t:t + 1], cache, state)
            ys.append(y)
    assert err(torch.cat(ys, 1), g["y"]) <= 1e-4
    assert err(state[0], g["states"][x.shape[1]]) <= 1e-4


@pytest.mark.parametrize("name", ["hofa_r16", "hofa_dh128_r32"])
@pytest.mark.parametrize("T0", [50, 64, 72])
def test_bf16_autocast_prefill_matches_reference(name, T0):
    g = load_golden(name)
    m = make_layer(g)
    x = g["x"].cuda()
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        y, cache, state = m(x[:, :T0].to(torch.bfloat16), return_state=True)
    assert y.dtype == torch.bfloat16
    assert err(y, g["y"][:, :T0]) <= 2e-2
    assert err(state[0], g["states"][T0]) <= 2e-2


def test_hybrid_prefill_eps_reproduces_the_inference_layer_choice():
    """The reference's inference layer normalises the hybrid prefill's GLA
    output with eps 1e-5 (src/chunk_gla_inlier.py:234), its training layer
    with float32 epsilon.  Small projections make the difference visible; the
    layer follows the oracle with either choice (float32)."""
    from outlierneuronattention_b200 import HybridOutlierFactorizedAttention, ModelConfig
    torch.manual_seed(0)
    m = HybridOutlierFactorizedAttention(ModelConfig(d_model=256, num_heads=4, num_layers=1, r=16, chunk_size=64))
    with torch.no_grad():
        m.gate_proj.weight.normal_(0, 0.02)
        m.mix_proj.weight.normal_(0, 0.02)
    sd = {k: v.clone() for k, v in m.state_dict().items()}
    x = torch.randn(2, 200, 256, generator=torch.Generator().manual_seed(4)) * 0.5
    m = m.cuda().eval()
    outs = {}
    for eps in (None, 1e-5):
        if eps is not None:
            m.hybrid_prefill_eps = eps
        ref = OracleLayer(LayerShape(256, 4, 16, 64), sd, **({} if eps is None else {"prefill_eps": eps}))
        with torch.no_grad():
            y = m(x.cuda())
        outs[eps] = y
        assert err(y, ref.forward(x.double())) <= 1e-4, eps
    assert err(outs[None], outs[1e-5]) > 1e-3   # the choice matters at this scale


def test_config0_fp32_against_oracle():
    """BASELINE config 0 shape (B=2, T=512, d_model=512, H=8, d_h=64, r=16,
    chunk 64) in float32, random gates and the outlier x8 weights."""
    from outlierneuronattention_b200 import HybridOutlierFactorizedAttention, ModelConfig
    torch.manual_seed(0)
    cfg = ModelConfig(d_model=512, num_heads=8, num_layers=1, r=16, chunk_size=64)
    m = HybridOutlierFactorizedAttention(cfg)
    gen = torch.Generator().manual_seed(0)
    with torch.no_grad():
        for lin in (m.W_q, m.W_k, m.W_v, m.out_proj):
            lin.weight.copy_(torch.randn(lin.weight.shape, generator=gen) * 0.02)
        for h in range(8):
            m.W_q.weight[h * 64:h * 64 + 16] *= 8
            m.W_k.weight[h * 64:h * 64 + 16] *= 8
        m.gate_proj.weight.copy_(torch.randn(m.gate_proj.weight.shape, generator=gen) * 0.02)
        m.mix_proj.weight.copy_(torch.randn(m.mix_proj.weight.shape, generator=gen) * 0.02)
    sd = {k: v.clone() for k, v in m.state_dict().items()}
    x = torch.randn(2, 512, 512, generator=gen)
    oracle = OracleLayer(LayerShape(512, 8, 16, 64), sd)
    ref_y, ref_cache, ref_state = oracle.forward(x.double(), return_state=True)
    m = m.cuda().eval()
    with torch.no_grad():
        y, cache, state = m(x.cuda(), return_state=True)
    assert err(y, ref_y) <= 1e-4
    assert err(cache[0], ref_cache[0]) <= 1e-4
    assert err(cache[1], ref_cache[1]) <= 1e-4
    assert err(state[0], ref_state) <= 1e-4
    # one more token through forward_step == the oracle's decode step
    xs = torch.randn(2, 1, 512, generator=gen)
    with torch.no_grad():
        ys, _, st2 = m.forward_step(xs.cuda(), cache, state)
    oy, _, ost = oracle.forward_step(xs.double(), ref_cache, ref_state)
    assert err(ys, oy) <= 1e-4
    assert err(st2[0], ost) <= 1e-4


def test_module_has_reference_parameter_names():
    from outlierneuronattention_b200 import HybridOutlierFactorizedAttention, ModelConfig
    g = load_golden("hofa_r16_alpha")
    m = make_layer(g)
    assert set(m.state_dict()) == set(g["state_dict"])


def test_no_rope_layer_prefill_export_and_preallocated_decode_fp32():
    """use_rope=False: the outlier cache holds un-rotated keys, written by the
    prefill export and by the fused decode step."""
    from outlierneuronattention_b200 import HybridOutlierFactorizedAttention, ModelConfig
    torch.manual_seed(1)
    cfg = ModelConfig(d_model=256, num_heads=4, num_layers=1, r=16, chunk_size=64, use_rope=False)
    m = HybridOutlierFactorizedAttention(cfg)
    gen = torch.Generator().manual_seed(1)
    with torch.no_grad():
        m.gate_proj.weight.copy_(torch.randn(m.gate_proj.weight.shape, generator=gen) * 0.02)
        m.mix_proj.weight.copy_(torch.randn(m.mix_proj.weight.shape, generator=gen) * 0.02)
    sd = {k: v.clone() for k, v in m.state_dict().items()}
    oracle = OracleLayer(LayerShape(256, 4, 16, 64, use_rope=False), sd)
    T0, T = 40, 48
    x = torch.randn(2, T, 256, generator=gen)
    ref_y, ref_cache, ref_state = oracle.forward(x[:, :T0].double(), return_state=True)
    m = m.cuda().eval()
    with torch.no_grad():
        y, cache, state = m(x[:, :T0].cuda(), return_state=True)
        assert err(y, ref_y) <= 1e-4 and err(cache[0], ref_cache[0]) <= 1e-4
        Kc = torch.zeros(2, 4, T, 16, device="cuda")
        Vc = torch.zeros(2, 4, T, 64, device="cuda")
        Kc[:, :, :T0], Vc[:, :, :T0] = cache
        cache = (Kc, Vc)
        oc, ost = ref_cache, ref_state
        for t in range(T0, T):
            ys, cache, state = m.forward_step(x[:, t:t + 1].cuda(), cache, state, cache_seq_len=t)
            oy, oc, ost = oracle.forward_step(x[:, t:t + 1].double(), oc, ost)
            assert err(ys, oy) <= 1e-4
    assert err(cache[0], oc[0]) <= 1e-4 and err(cache[1], oc[1]) <= 1e-4
    assert err(state[0], ost) <= 1e-4


def test_device_position_decode_loop_in_cuda_graph():
    """forward_step with cache_seq_len as an int32 CUDA scalar: two decode steps
    (state ping-pong, position advanced on the device) captured once and
    replayed eight times give the eager host-position loop's outputs."""
    from outlierneuronattention_b200 import HybridOutlierFactorizedAttention, ModelConfig
    torch.manual_seed(2)
    cfg = ModelConfig(d_model=256, num_heads=4, num_layers=1, r=16, chunk_size=64)
    m = HybridOutlierFactorizedAttention(cfg)
    gen = torch.Generator().manual_seed(2)
    with torch.no_grad():
        m.gate_proj.weight.copy_(torch.randn(m.gate_proj.weight.shape, generator=gen) * 0.02)
        m.mix_proj.weight.copy_(torch.randn(m.mix_proj.weight.shape, generator=gen) * 0.02)
    m = m.cuda().eval()
    T0, NS, CAP = 37, 16, 64
    x = torch.randn(2, T0 + NS, 256, generator=gen).cuda()

    def prefill():
        _, (k, v), (s, _) = m(x[:, :T0], return_state=True)
        K = torch.zeros(2, 4, CAP, 16, device="cuda")
        V = torch.zeros(2, 4, CAP, 64, device="cuda")
        K[:, :, :T0], V[:, :, :T0] = k, v
        return (K, V), s.clone(), torch.empty_like(s)

    with torch.no_grad():
        cache, sa, sb = prefill()
        ref, state = [], (sa, sb)
        for t in range(T0, T0 + NS):
            y, cache, state = m.forward_step(x[:, t:t + 1], cache, state, cache_seq_len=t)
            ref.append(y.clone())
        ref_cache, ref_state = cache, state[0]

        cache, sa, sb = prefill()
        pos = torch.tensor([T0], dtype=torch.int32, device="cuda")
        xb = [x[:, T0:T0 + 1].clone(), x[:, T0 + 1:T0 + 2].clone()]
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            # warm-up on scratch copies (creates the layer's cached buffers), then capture
            wc = (cache[0].clone(), cache[1].clone())
            wp = pos.clone()
            m.forward_step(xb[0], wc, (sa.clone(), sb.clone()), cache_seq_len=wp)
            s.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                y0, _, _ = m.forward_step(xb[0], cache, (sa, sb), cache_seq_len=pos)
                pos.add_(1)
                y1, _, _ = m.forward_step(xb[1], cache, (sb, sa), cache_seq_len=pos)
                pos.add_(1)
            out = []
            for i in range(NS // 2):
                xb[0].copy_(x[:, T0 + 2 * i:T0 + 2 * i + 1])
                xb[1].copy_(x[:, T0 + 2 * i + 1:T0 + 2 * i + 2])
                g.replay()
                out += [y0.clone(), y1.clone()]
            s.synchronize()
        del g
    for a, b in zip(out, ref):
        assert err(a, b) <= 1e-4
    assert int(pos.item()) == T0 + NS
    assert err(cache[0], ref_cache[0]) <= 1e-5 and err(cache[1], ref_cache[1]) <= 1e-5
    assert err(sa, ref_state) <= 1e-4
