"""Pin the CPU oracle against the reference's own outputs.

The fixtures in ``tests/golden`` are outputs of the reference layer
``HybridOutlierFactorizedAttentionTrain.forward_step``
(src/HybridOutlierFactorizedAttentionTrain.py:298-438), run token by token in
float64 by ``tests/golden/make_golden.py``.  The oracle must reproduce them
both token by token (its decode restatement) and in one prefill call (its
chunked-GLA + causal-attention restatement).
"""
import pytest
import torch

from conftest import GOLDEN_CASES, load_golden
from oracle.hofa_oracle import (LayerShape, OracleLayer, chunk_gla_core, chunk_gla_reference_rounding,
                                outlier_attention_core, decode_core)

TOL = 2e-6  # fixtures are stored in fp32


def _layer(g, gla_mode="chunk"):
    c = g["config"]
    shape = LayerShape(d_model=c["d_model"], num_heads=c["num_heads"], r=c["r"],
                       chunk_size=c["chunk_size"], rope_base=c["rope_base"], use_rope=c["use_rope"])
    return OracleLayer(shape, g["state_dict"], gla_mode=gla_mode)


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_oracle_decode_loop_matches_reference(name):
    g = load_golden(name)
    layer = _layer(g)
    x = g["x"].double()
    T = x.shape[1]
    cache, state = None, None
    ys = []
    for t in range(T):
        y, cache, state = layer.forward_step(x[:, t:t + 1], cache, state)
        ys.append(y)
        if t + 1 in g["states"]:
            torch.testing.assert_close(state.float(), g["states"][t + 1], atol=TOL, rtol=1e-5)
    torch.testing.assert_close(torch.cat(ys, 1).float(), g["y"], atol=TOL, rtol=1e-5)
    if g["cache_k"] is not None:
        torch.testing.assert_close(cache[0].float(), g["cache_k"], atol=TOL, rtol=1e-5)
        torch.testing.assert_close(cache[1].float(), g["cache_v"], atol=TOL, rtol=1e-5)


@pytest.mark.parametrize("name", GOLDEN_CASES)
@pytest.mark.parametrize("gla_mode", ["chunk", "recurrent"])
def test_oracle_prefill_matches_reference(name, gla_mode):
    g = load_golden(name)
    layer = _layer(g, gla_mode)
    x = g["x"].double()
    for T0 in sorted(g["states"]):
        out, cache, state = layer.forward(x[:, :T0], return_state=True)
        torch.testing.assert_close(out.float(), g["y"][:, :T0], atol=TOL, rtol=1e-5)
        torch.testing.assert_close(state.float(), g["states"][T0], atol=TOL, rtol=1e-5)
        if cache is not None:
            torch.testing.assert_close(cache[0].float(), g["cache_k"][:, :, :T0], atol=TOL, rtol=1e-5)
            torch.testing.assert_close(cache[1].float(), g["cache_v"][:, :, :T0], atol=TOL, rtol=1e-5)


def test_oracle_prefill_then_decode_matches_reference():
    """Prefill 50 tokens, then decode the rest on the exported cache/state."""
    g = load_golden("hofa_r16")
    layer = _layer(g)
    x = g["x"].double()
    out, cache, state = layer.forward(x[:, :50], return_state=True)
    ys = [out]
    for t in range(50, x.shape[1]):
        y, cache, state = layer.forward_step(x[:, t:t + 1], cache, state)
        ys.append(y)
    torch.testing.assert_close(torch.cat(ys, 1).float(), g["y"], atol=TOL, rtol=1e-5)


def test_chunk_forms_agree_with_alpha_and_ragged_chunks():
    gen = torch.Generator().manual_seed(3)
    B, H, T, D, r = 2, 3, 150, 64, 16
    Q, K, V = (torch.randn(B, H, T, D, generator=gen, dtype=torch.float64) * 0.5 for _ in range(3))
    lg = torch.nn.functional.logsigmoid(torch.randn(B, H, T, generator=gen, dtype=torch.float64))
    la = torch.randn(1, H, 1, D - r, generator=gen, dtype=torch.float64) * 0.5
    mix = torch.rand(B, H, T, generator=gen, dtype=torch.float64)
    gs = torch.randn(1, H, 1, D, generator=gen, dtype=torch.float64)
    s0 = torch.randn(B, H, D - r, D, generator=gen, dtype=torch.float64)
    for alpha in (None, la):
        a = chunk_gla_core(Q, K, V, lg, r, 64, alpha, mix, gs, state_init=s0)
        b = chunk_gla_core(Q, K, V, lg, r, 64, alpha, mix, gs, state_init=s0, mode="recurrent")
        c = chunk_gla_core(Q, K, V, lg, r, 32, alpha, mix, gs, state_init=s0)
        for u, w in ((a, b), (a, c)):
            torch.testing.assert_close(u[0], w[0], atol=1e-10, rtol=1e-9)
            torch.testing.assert_close(u[1], w[1], atol=1e-10, rtol=1e-9)


def test_reference_rounding_form_is_the_chunk_form_in_float64():
    """The restatement of the reference kernel's rounding points reduces to the
    float64 chunk form when the inputs are float64 (every rounding is then the
    identity), with and without a per-channel decay, and on bf16 inputs stays
    within bf16 rounding of it."""
    gen = torch.Generator().manual_seed(4)
    B, H, T, D, r = 1, 2, 200, 64, 16
    Q, K, V = (torch.randn(B, H, T, D, generator=gen, dtype=torch.float64) * 0.3 for _ in range(3))
    lg = torch.nn.functional.logsigmoid(torch.randn(B, H, T, generator=gen, dtype=torch.float64) + 3.0)
    la = torch.randn(1, H, 1, D - r, generator=gen, dtype=torch.float64) * 0.5
    mix = torch.rand(B, H, T, generator=gen, dtype=torch.float64)
    gs = torch.randn(1, H, 1, D, generator=gen, dtype=torch.float64)
    for alpha in (None, la):
        a = chunk_gla_core(Q, K, V, lg, r, 64, alpha, mix, gs)
        b = chunk_gla_reference_rounding(Q, K, V, lg, r, 64, alpha, mix, gs)
        torch.testing.assert_close(a[0], b[0], atol=1e-12, rtol=1e-10)
        torch.testing.assert_close(a[1], b[1], atol=1e-12, rtol=1e-10)
        c = chunk_gla_reference_rounding(Q.bfloat16(), K.bfloat16(), V.bfloat16(), lg, r, 64, alpha, mix, gs)
        d = chunk_gla_core(Q.bfloat16(), K.bfloat16(), V.bfloat16(), lg, r, 64, alpha, mix, gs)
        assert 0 < (c[0] - d[0]).abs().max().item() < 5e-2


def test_outlier_attention_q_offset_equals_suffix_of_full():
    """A query shard with q_offset sees exactly the rows the full causal call sees."""
    gen = torch.Generator().manual_seed(4)
    B, H, T, D, r = 1, 2, 96, 64, 16
    Q, K, V = (torch.randn(B, H, T, D, generator=gen, dtype=torch.float64) for _ in range(3))
    mix = torch.rand(B, H, T, generator=gen, dtype=torch.float64)
    full = outlier_attention_core(Q, K, V, r, 2.0, mix)
    part = outlier_attention_core(Q[:, :, 40:], K, V, r, 2.0, mix[:, :, 40:], q_offset=40)
    torch.testing.assert_close(part, full[:, :, 40:], atol=1e-12, rtol=1e-12)


def test_decode_core_equals_one_step_of_prefill():
    """decode at position p == the last row of a causal prefill of p+1 tokens."""
    gen = torch.Generator().manual_seed(5)
    B, H, T, D, r = 2, 2, 33, 64, 16
    Q, K, V = (torch.randn(B, H, T, D, generator=gen, dtype=torch.float64) for _ in range(3))
    lg = torch.nn.functional.logsigmoid(torch.randn(B, H, T, generator=gen, dtype=torch.float64))
    mix = torch.rand(B, H, T, generator=gen, dtype=torch.float64)
    gs = torch.randn(H, D, generator=gen, dtype=torch.float64)
    from oracle.hofa_oracle import FP32_EPS
    Y, S = chunk_gla_core(Q, K, V, lg, r, 16, None, mix, gs, eps=FP32_EPS)
    Y = outlier_attention_core(Q, K, V, r, 2.0, mix, out=Y)
    _, S_prev = chunk_gla_core(Q[:, :, :-1], K[:, :, :-1], V[:, :, :-1], lg[:, :, :-1], r, 16)
    y, S_new = decode_core(Q[:, :, -1:], K[:, :, -1:], V[:, :, -1:], K[:, :, :, :r], V, S_prev,
                           lg[:, :, -1:], mix[:, :, -1:], gs, r, T, 2.0)
    torch.testing.assert_close(y, Y[:, :, -1:], atol=1e-12, rtol=1e-10)
    torch.testing.assert_close(S_new, S, atol=1e-12, rtol=1e-10)
