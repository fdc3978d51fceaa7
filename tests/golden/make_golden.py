"""Generate the golden fixtures ``tests/golden/*.pt`` from the reference itself.

Runs the reference's own PyTorch layer,
``HybridOutlierFactorizedAttentionTrain.forward_step``
(src/HybridOutlierFactorizedAttentionTrain.py:298-438 of
LotanGutman/OutlierNeuronAttention), token by token on CPU in float64.  A
token-by-token ``forward_step`` loop is the reference's pure-PyTorch prefill
(no substitution of its Triton/``fla`` dependencies is needed), and its last
steps are ordinary decode steps.

Two ablation branches have their own fixtures: ``r == d_head`` (plain
attention) from the same training layer's ``forward_step``, and the width
split (``mha_heads_for_width_split``: softmax heads beside GLA heads) from the
inference layer's ``forward_step``
(src/HybridOutlierFactorizedAttention.py:234-296), whose width-split decode
is plain PyTorch (the training layer has no width-split decode).

Needs the path of a reference checkout (``--ref``, required), so it runs only
where that checkout exists; the GPU box never runs it.  The
fixtures it writes are small and self-contained: weights, input, per-token
outputs, the final outlier cache and GLA states at a few prefix lengths.

    python tests/golden/make_golden.py --ref PATH [--only NAME ...]
"""
from __future__ import annotations

import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# name: (ModelConfig overrides, B, T)
CASES = {
    "hofa_r16": (dict(d_model=128, num_heads=2, r=16), 2, 72),
    "hofa_r16_alpha": (dict(d_model=64, num_heads=1, r=16, learnable_alpha=True), 2, 72),
    "hofa_r16_fixedmix": (dict(d_model=64, num_heads=1, r=16, fixed_blend_weight=True), 2, 72),
    "hofa_dh128_r32": (dict(d_model=128, num_heads=1, r=32), 2, 72),
    "gla_r0": (dict(d_model=64, num_heads=1, r=0), 2, 72),
    "mha_r_eq_dh": (dict(d_model=128, num_heads=2, r=64), 2, 72),
    "width_split": (dict(d_model=192, num_heads=3, r=0, mha_heads_for_width_split=1), 2, 72),
}
# cases run through the inference layer (the training layer lacks their decode branch)
INFERENCE_LAYER_CASES = {"width_split"}
CHECKPOINTS = (50, 64)


def make_case(name, over, B, T, ModelConfig, HOFA, tuple_state=False):
    torch.manual_seed(1234 + sum(map(ord, name)))
    cfg = ModelConfig(num_layers=1, chunk_size=64, use_rope=True, mix_gate_bias_init=0.0, **over)
    m = HOFA(cfg)
    H, D, r = cfg.num_heads, cfg.d_model // cfg.num_heads, cfg.r
    g = torch.Generator().manual_seed(7 + len(name))
    with torch.no_grad():
        for lin in (m.W_q, m.W_k, m.W_v, m.out_proj):
            lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) * 0.02)
        # "outlier x8": the first r channels of every head carry heavy-tailed q/k
        for h in range(H):
            m.W_q.weight[h * D:h * D + r] *= 8.0
            m.W_k.weight[h * D:h * D + r] *= 8.0
        m.gate_proj.weight.copy_(torch.randn(m.gate_proj.weight.shape, generator=g) * 0.5)
        m.gate_proj.bias.copy_(torch.randn(m.gate_proj.bias.shape, generator=g) * 0.5 - 1.0)
        if hasattr(m, "mix_proj"):
            m.mix_proj.weight.copy_(torch.randn(m.mix_proj.weight.shape, generator=g) * 0.5)
            m.mix_proj.bias.copy_(torch.randn(m.mix_proj.bias.shape, generator=g) * 0.5)
        if hasattr(m, "fixed_mix"):
            m.fixed_mix.copy_(torch.randn(m.fixed_mix.shape, generator=g))
        if hasattr(m, "log_alpha"):
            m.log_alpha.copy_(torch.randn(m.log_alpha.shape, generator=g) * 0.5)
        m.gla_scale.copy_(1.0 + 0.2 * torch.randn(m.gla_scale.shape, generator=g))
        # weights are stored in fp32; the reference runs on exactly those values
        for p in m.parameters():
            p.copy_(p.float())
    sd = {k: v.detach().float().clone() for k, v in m.state_dict().items()}
    # the inference layer's width-split decode casts q/k/v to float32 itself
    # (src/HybridOutlierFactorizedAttention.py:279-281), so it runs in float32
    run_dtype = torch.float32 if tuple_state else torch.float64
    m = m.to(run_dtype).eval()
    x = torch.randn(B, T, cfg.d_model, generator=g).float()
    ys, states = [], {}
    cache, state = None, None
    with torch.no_grad():
        for t in range(T):
            y, cache, state = m.forward_step(x[:, t:t + 1].to(run_dtype), cache, state)
            ys.append(y.float())
            S = state[0] if tuple_state else state   # the inference layer returns (state_out, state_in)
            if S is not None and (t + 1 in CHECKPOINTS or t + 1 == T):
                states[t + 1] = S[:, :, :D - r, :].float().clone()
    out = {
        "name": name,
        "config": dict(d_model=cfg.d_model, num_heads=H, r=r, chunk_size=cfg.chunk_size,
                       learnable_alpha=cfg.learnable_alpha, fixed_blend_weight=cfg.fixed_blend_weight,
                       use_rope=cfg.use_rope, rope_base=cfg.rope_base, mix_gate_bias_init=cfg.mix_gate_bias_init,
                       mha_heads_for_width_split=cfg.mha_heads_for_width_split),
        "state_dict": sd,
        "x": x,
        "y": torch.cat(ys, dim=1),
        "states": states,
        "cache_k": None if cache is None else cache[0].float().contiguous(),
        "cache_v": None if cache is None else cache[1].float().contiguous(),
        "generator": ("tests/golden/make_golden.py: " + ("HybridOutlierFactorizedAttention.forward_step, float32"
                      if tuple_state else "HybridOutlierFactorizedAttentionTrain.forward_step, float64") + ", CPU"),
    }
    torch.save(out, os.path.join(HERE, f"{name}.pt"))
    print(f"{name}: B={B} T={T} H={H} D={D} r={r} |y|max={out['y'].abs().max():.3f}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of a LotanGutman/OutlierNeuronAttention checkout")
    ap.add_argument("--only", nargs="*", default=None, help="regenerate only these cases")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    from src.config import ModelConfig
    from src.HybridOutlierFactorizedAttention import HybridOutlierFactorizedAttention as HOFAInfer
    from src.HybridOutlierFactorizedAttentionTrain import HybridOutlierFactorizedAttention as HOFA
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name, (over, B, T) in CASES.items():
        if args.only and name not in args.only:
            continue
        infer = name in INFERENCE_LAYER_CASES
        make_case(name, over, B, T, ModelConfig, HOFAInfer if infer else HOFA, tuple_state=infer)


if __name__ == "__main__":
    main()
