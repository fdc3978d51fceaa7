"""CPU oracle for the HOFA attention hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path (the package
``outlierneuronattention_b200``) imports this module.  It is used by
``tests/`` as the checker, by ``__graft_entry__.smoke()`` as the checker and
by ``bench.py`` for the CPU baseline leg (``cpu_baseline`` /
``--impl reference``).

It restates, in plain PyTorch CPU arithmetic, the reference algorithm of
LotanGutman/OutlierNeuronAttention for the Hybrid Outlier-Factorized
Attention (HOFA) layer:

* ``decode_core``      -- ``fused_hofa_decode``       (src/hofa_decode_triton.py:342-476,
                                                         kernels :47-159, :172-340)
* ``chunk_gla_core``   -- ``chunk_gla_inlier_fwd``     (src/chunk_gla_inlier.py:153-237,
                                                         kernel :5-150)
* ``outlier_attention_core`` -- ``exact_attention_triton`` (src/exact_attention.py:163-188,
                                                         kernel :45-161)
* ``OracleLayer.forward`` / ``forward_step`` -- the training module's layer
  (src/HybridOutlierFactorizedAttentionTrain.py:128-296 and :298-438), which
  is the reference's own PyTorch implementation of the layer.

Parity pin: ``tests/golden/*.pt`` hold outputs of the reference's own
``HybridOutlierFactorizedAttentionTrain.forward_step`` run token by token on
CPU in float64 (generator: ``tests/golden/make_golden.py``), and
``tests/test_oracle_golden.py`` checks this oracle against them.

By default everything runs in float64.  ``act_dtype`` rounds the projected
activations to the activation dtype (bf16) the way a bf16 model does, so the
oracle sees the same bf16-rounded inputs as the GPU kernels.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

FP32_EPS = float(torch.finfo(torch.float32).eps)


# --------------------------------------------------------------------------
# RoPE -- src/modules/modules.py:5-45
# --------------------------------------------------------------------------
def rope_cos_sin(dim: int, n: int, base: float = 10000.0,
                 dtype=torch.float64) -> Tuple[torch.Tensor, torch.Tensor]:
    """cos/sin tables of ``RotaryEmbedding`` (modules.py:9-17): inv_freq is
    computed in fp32, the angle table ``outer(t, inv_freq)`` in fp32, then
    cos/sin; rows are positions, columns ``cat(freqs, freqs)``."""
    inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    t = torch.arange(n, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """modules.py:33-36."""
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """modules.py:38-45 for one tensor; cos/sin are [N, d] and broadcast over (B, H)."""
    return x * cos + rotate_half(x) * sin


# --------------------------------------------------------------------------
# Operator-level oracles
# --------------------------------------------------------------------------
def _gamma_rows(log_gamma: torch.Tensor, J: int,
                log_alpha: Optional[torch.Tensor]) -> torch.Tensor:
    """Per-row decay of the GLA state for one token.

    log_gamma: [B, H]; returns [B, H, J, 1].  Without ``log_alpha`` every row
    decays by exp(log_gamma) (hofa_decode_triton.py:88); with it row c decays
    by exp(log_gamma * exp(log_alpha_c)) (hofa_decode_triton.py:103-106)."""
    B, H = log_gamma.shape
    if log_alpha is None:
        return torch.exp(log_gamma).view(B, H, 1, 1).expand(B, H, J, 1)
    a = torch.exp(log_alpha.reshape(-1, H, J).to(log_gamma.dtype))  # [1|B, H, J]
    return torch.exp(log_gamma.view(B, H, 1) * a).view(B, H, J, 1)


def decode_core(q, k, v, cache_k, cache_v, state_in, log_gamma, mix_g, norm_w,
                R: int, seq_len: int, sm_scale: float,
                log_alpha=None, eps: float = FP32_EPS,
                dtype=torch.float64):
    """One HOFA decode step of the attention core.

    Restates ``fused_hofa_decode`` (src/hofa_decode_triton.py:342-476): the
    GLA update ``S' = gamma*S + k_I v^T`` and inclusive readout
    ``y_I = q_I S'`` (kernel :93-114), the softmax of ``q_O . K_cache[t]`` over
    the first ``seq_len`` cache rows (:128-151, split form :211-231 combined at
    :306-330), RMSNorm(y_I) * norm_w (:153-156) and the blend
    ``mix*y_O + (1-mix)*y_I_norm`` (:158).

    Shapes: q,k,v [B,H,1,D]; cache_k [B,H,L>=seq_len,R]; cache_v
    [B,H,L,D]; state_in [B,H,J,D]; log_gamma, mix_g [B,H,1] (or [B,H]);
    norm_w [H,D].  Returns (Y [B,H,1,D], state_out [B,H,J,D]) in ``dtype``.
    """
    B, H, _, D = q.shape
    J = D - R
    f = lambda t: t.to(dtype)
    q, k, v = f(q)[:, :, 0], f(k)[:, :, 0], f(v)[:, :, 0]
    lg = f(log_gamma).reshape(B, H)
    mg = f(mix_g).reshape(B, H)
    S = f(state_in)
    g = _gamma_rows(lg, J, None if log_alpha is None else f(log_alpha))
    S_new = g * S + k[:, :, R:, None] * v[:, :, None, :]
    y_i = torch.einsum('bhj,bhjd->bhd', q[:, :, R:], S_new)
    if R > 0:
        Kc = f(cache_k[:, :, :seq_len, :R])
        Vc = f(cache_v[:, :, :seq_len, :])
        s = torch.einsum('bhr,bhtr->bht', q[:, :, :R], Kc) * sm_scale
        p = torch.softmax(s, dim=-1)
        y_o = torch.einsum('bht,bhtd->bhd', p, Vc)
    else:
        y_o = torch.zeros_like(y_i)
    var = (y_i * y_i).mean(-1, keepdim=True)
    y_n = y_i * torch.rsqrt(var + eps) * f(norm_w).reshape(1, H, D)
    y = mg[..., None] * y_o + (1.0 - mg[..., None]) * y_n
    return y[:, :, None, :], S_new


def chunk_gla_core(Q, K, V, log_gamma, r: int, chunk_size: int = 64,
                   log_alpha=None, mix_g=None, gla_scale=None,
                   eps: float = 1e-5, state_init=None,
                   dtype=torch.float64, mode: str = "chunk"):
    """Gated linear attention over the inlier channels ``[r:D]`` of Q/K.

    Restates ``chunk_gla_inlier_fwd`` (src/chunk_gla_inlier.py:153-237).  The
    recurrence is ``S_t = diag(gamma_t) S_{t-1} + k_t v_t^T``, ``y_t = q_t S_t``
    (inclusive), computed chunk by chunk as in the kernel (:86-126):
    ``Y = ((Q K^T) * exp(G_i - G_j) [i>=j]) V + (Q S_prev) * exp(G_i)`` and
    ``S <- exp(G_C) S_prev + (K * exp(G_C - G_j))^T V``, where G is the
    in-chunk cumulative sum of the log decay (per channel when ``log_alpha``
    is given, :90-107).  When both ``mix_g`` and ``gla_scale`` are given the
    output is ``(1 - mix) * gla_scale * RMSNorm(y)`` (:130-141), otherwise the
    raw ``y``.

    ``mode="recurrent"`` evaluates the same function token by token (used by
    the tests to cross-check the chunk algebra).  ``state_init`` ([B,H,J,D])
    seeds S_0 (zero in the reference; used by sequence-sharded prefill).
    Returns (Y [B,H,T,D], S_T [B,H,J,D]).
    """
    B, H, T, D = Q.shape
    J = D - r
    f = lambda t: t.to(dtype)
    q = f(Q[..., r:])
    kk = f(K[..., r:])
    vv = f(V)
    lg = f(log_gamma).reshape(B, H, T)
    if log_alpha is not None:
        alpha = torch.exp(f(log_alpha).reshape(-1, H, J))[:, :, None, :]  # [.,H,1,J]
        g = lg[..., None] * alpha                                           # [B,H,T,J]
    else:
        g = lg[..., None].expand(B, H, T, J)
    S = torch.zeros(B, H, J, D, dtype=dtype) if state_init is None else f(state_init).clone()
    Y = torch.empty(B, H, T, D, dtype=dtype)
    if mode == "recurrent":
        for t in range(T):
            S = torch.exp(g[:, :, t, :, None]) * S + kk[:, :, t, :, None] * vv[:, :, t, None, :]
            Y[:, :, t] = torch.einsum('bhj,bhjd->bhd', q[:, :, t], S)
    else:
        for s0 in range(0, T, chunk_size):
            s1 = min(T, s0 + chunk_size)
            qc, kc, vc, gc = q[:, :, s0:s1], kk[:, :, s0:s1], vv[:, :, s0:s1], g[:, :, s0:s1]
            G = torch.cumsum(gc, dim=2)                                    # [B,H,C,J]
            C = s1 - s0
            diff = G[:, :, :, None, :] - G[:, :, None, :, :]               # [B,H,C,C,J]
            causal = torch.tril(torch.ones(C, C, dtype=torch.bool))
            w = torch.where(causal[None, None, :, :, None], torch.exp(diff.clamp(max=0.0)),
                            torch.zeros((), dtype=dtype))
            attn = torch.einsum('bhij,bhsj,bhisj->bhis', qc, kc, w)
            y_intra = attn @ vc
            y_inter = (qc * torch.exp(G)) @ S
            Y[:, :, s0:s1] = y_intra + y_inter
            GC = G[:, :, -1, :]                                            # [B,H,J]
            kd = kc * torch.exp(GC[:, :, None, :] - G)
            S = torch.exp(GC)[..., None] * S + kd.transpose(-1, -2) @ vc
    if mix_g is not None and gla_scale is not None:
        var = (Y * Y).mean(-1, keepdim=True)
        Y = Y * torch.rsqrt(var + eps) * f(gla_scale).reshape(1, H, 1, D)
        Y = Y * (1.0 - f(mix_g).reshape(B, H, T, 1))
    return Y, S


def chunk_gla_reference_rounding(Q, K, V, log_gamma, r: int, chunk_size: int = 64, log_alpha=None,
                                 mix_g=None, gla_scale=None, eps: float = 1e-5, state_init=None):
    """``chunk_gla_fwd_kernel`` (src/chunk_gla_inlier.py:5-150) with its rounding
    points: the same chunk loop as ``chunk_gla_core`` in float64, but every
    operand the reference casts to the input dtype before a ``tl.dot`` is
    rounded to it here -- with a per-channel decay (``HAS_ALPHA``, :90-107) the
    factored queries and keys, the masked score matrix, the decayed queries of
    the inter-chunk term and the carried state; with a scalar decay (:108-126)
    the masked score matrix, the carried state and the decayed keys.  The
    output is rounded to the input dtype at the end (:143-144).  Used by the
    tests as the reference's own error against the float64 ``chunk_gla_core``
    on the same inputs.  Returns (Y [B,H,T,D] float64, S_T [B,H,J,D]).
    """
    B, H, T, D = Q.shape
    J = D - r
    lowp = Q.dtype
    f = lambda t: t.to(torch.float64)
    rnd = lambda t: t.to(lowp).to(torch.float64)
    q, kk, vv = f(Q[..., r:]), f(K[..., r:]), f(V)
    lg = f(log_gamma).reshape(B, H, T)
    alpha = torch.exp(f(log_alpha).reshape(-1, H, J))[:, :, None, :] if log_alpha is not None else None
    S = torch.zeros(B, H, J, D, dtype=torch.float64) if state_init is None else f(state_init).clone()
    Y = torch.empty(B, H, T, D, dtype=torch.float64)
    for s0 in range(0, T, chunk_size):
        s1 = min(T, s0 + chunk_size)
        C = s1 - s0
        qc, kc, vc = q[:, :, s0:s1], kk[:, :, s0:s1], vv[:, :, s0:s1]
        G = torch.cumsum(lg[:, :, s0:s1], dim=2)                               # [B,H,C]
        GL = G[:, :, -1:]
        causal = torch.tril(torch.ones(C, C, dtype=torch.bool))
        if alpha is not None:
            qf = rnd(qc * torch.exp((G - GL)[..., None] * alpha))
            kf = rnd(kc * torch.exp((GL - G)[..., None] * alpha))
            attn = rnd(torch.where(causal, qf @ kf.transpose(-1, -2), torch.zeros((), dtype=torch.float64)))
            y_intra = attn @ vc
            y_inter = rnd(qc * torch.exp(G[..., None] * alpha)) @ rnd(S)
            S = S * torch.exp(GL[..., None] * alpha).transpose(-1, -2) + kf.transpose(-1, -2) @ vc
        else:
            mask = torch.where(causal, torch.exp((G[..., :, None] - G[..., None, :]).clamp(max=0.0)),
                               torch.zeros((), dtype=torch.float64))
            attn = rnd((qc @ kc.transpose(-1, -2)) * mask)
            y_intra = attn @ vc
            y_inter = (qc @ rnd(S)) * torch.exp(G)[..., None]
            kd = rnd(kc * torch.exp(GL - G)[..., None])
            S = S * torch.exp(GL)[..., None] + kd.transpose(-1, -2) @ vc
        Y[:, :, s0:s1] = y_intra + y_inter
    if mix_g is not None and gla_scale is not None:
        var = (Y * Y).mean(-1, keepdim=True)
        Y = Y * torch.rsqrt(var + eps) * f(gla_scale).reshape(1, H, 1, D)
        Y = Y * (1.0 - f(mix_g).reshape(B, H, T, 1))
    return rnd(Y), S


def outlier_attention_core(Q, K, V, r: int, sm_scale: float, mix_g, out=None,
                           q_offset: int = 0, dtype=torch.float64, block: int = 256):
    """Causal softmax attention over the first ``r`` channels of Q/K with
    full-width V, scaled by ``mix_g`` and added into ``out``.

    Restates ``exact_attention_triton`` (src/exact_attention.py:163-188) and
    its kernel (:45-161): ``out += mix * softmax(sm_scale * Q_r K_r^T, causal) V``
    (the add-in-place is :153-161).  Key j is visible to query i when
    ``j <= i + q_offset`` (the reference has q_offset = 0; a query shard of a
    sequence-sharded prefill uses the absolute position of its first row).
    Returns the updated ``out`` (a new tensor in ``dtype``).
    """
    B, H, Tq = Q.shape[:3]
    Tk, D = K.shape[2], V.shape[-1]
    f = lambda t: t.to(dtype)
    qr, kr, vv = f(Q[..., :r]), f(K[..., :r]), f(V)
    mg = f(mix_g).reshape(B, H, Tq)
    res = torch.zeros(B, H, Tq, D, dtype=dtype) if out is None else f(out).clone()
    kpos = torch.arange(Tk)
    for i0 in range(0, Tq, block):
        i1 = min(Tq, i0 + block)
        s = torch.einsum('bhir,bhjr->bhij', qr[:, :, i0:i1], kr) * sm_scale
        qpos = torch.arange(i0, i1) + q_offset
        s = s.masked_fill(kpos[None, :] > qpos[:, None], float('-inf'))
        p = torch.softmax(s, dim=-1)
        res[:, :, i0:i1] += mg[:, :, i0:i1, None] * (p @ vv)
    return res


# --------------------------------------------------------------------------
# Layer-level oracle: HybridOutlierFactorizedAttentionTrain
# --------------------------------------------------------------------------
@dataclass
class LayerShape:
    d_model: int
    num_heads: int
    r: int
    chunk_size: int = 64
    rope_base: float = 10000.0
    use_rope: bool = True
    attention_scale: float = 1.0

    @property
    def d_head(self) -> int:
        return self.d_model // self.num_heads

    @property
    def j(self) -> int:
        return self.d_head - self.r


class OracleLayer:
    """The HOFA layer computed from a reference state dict.

    Parameter names are the reference's (HybridOutlierFactorizedAttentionTrain.py:29-72):
    ``W_q.weight, W_k.weight, W_v.weight, out_proj.weight, gate_proj.{weight,bias},
    mix_proj.{weight,bias} | fixed_mix, log_alpha (optional), gla_scale``.
    """

    def __init__(self, shape: LayerShape, state_dict: dict, dtype=torch.float64,
                 act_dtype=None, gla_mode: str = "chunk", prefill_eps: float = FP32_EPS):
        self.s = shape
        self.dtype = dtype
        # RMSNorm epsilon of the hybrid prefill: float32 epsilon in the training
        # layer (Train.py:71); the inference layer's Triton prefill uses 1e-5
        # (src/chunk_gla_inlier.py:234)
        self.prefill_eps = prefill_eps
        self.act_dtype = act_dtype
        self.gla_mode = gla_mode
        self.p = {k: v.detach().to(dtype) for k, v in state_dict.items()
                  if torch.is_tensor(v) and k.split('.')[0] != 'rotary_emb'}

    # -- helpers ----------------------------------------------------------
    def _act(self, t):
        if self.act_dtype is None:
            return t
        return t.to(self.act_dtype).to(self.dtype)

    def _proj(self, x):
        """Q, K, V projections, Train.py:130-137 / :302-307."""
        B, N, _ = x.shape
        s = self.s
        x = x.to(self.dtype)
        sf = s.d_head ** 0.25
        Q = self._act(x @ self.p['W_q.weight'].T / sf).view(B, N, s.num_heads, s.d_head).transpose(1, 2)
        K = self._act(x @ self.p['W_k.weight'].T / sf).view(B, N, s.num_heads, s.d_head).transpose(1, 2)
        V = self._act(x @ self.p['W_v.weight'].T).view(B, N, s.num_heads, s.d_head).transpose(1, 2)
        return Q, K, V

    def gates(self, Q, K):
        """``_compute_gates_optimized`` (Train.py:85-113): gate logits and the
        sigmoid mixing gate from the un-rotated full Q, K."""
        s = self.s
        D = s.d_head
        Wg = self.p['gate_proj.weight']
        bg = self.p['gate_proj.bias'].view(1, s.num_heads, 1)
        logits = torch.einsum('bhnf,hf->bhn', Q, Wg[:, :D]) + torch.einsum('bhnf,hf->bhn', K, Wg[:, D:]) + bg
        if 'mix_proj.weight' in self.p:
            Wm = self.p['mix_proj.weight']
            bm = self.p['mix_proj.bias'].view(1, s.num_heads, 1)
            ml = torch.einsum('bhnf,hf->bhn', Q, Wm[:, :D]) + torch.einsum('bhnf,hf->bhn', K, Wm[:, D:]) + bm
            mix = self._act(torch.sigmoid(ml))
        elif 'fixed_mix' in self.p:
            mix = self._act(torch.sigmoid(self.p['fixed_mix'])).reshape(1, s.num_heads, 1).expand(Q.shape[0], -1, Q.shape[2])
        else:
            mix = None
        return logits, mix

    def _log_alpha(self):
        return self.p.get('log_alpha')

    def _out(self, Y):
        B, H, N, D = Y.shape
        Y = Y.transpose(1, 2).reshape(B, N, H * D)
        return Y @ self.p['out_proj.weight'].T

    # -- prefill: Train.forward (:233-296) ----------------------------------
    def forward(self, x, return_state: bool = False):
        """Hybrid branch of Train.forward.  Returns the layer output and, when
        ``return_state``, the inference-module cache layout
        ``(K_O rotated [B,H,N,r], V [B,H,N,D])`` and GLA state ``[B,H,j,D]``."""
        s = self.s
        B, N, _ = x.shape
        Q, K, V = self._proj(x)
        logits, mix = self.gates(Q, K)
        log_gamma = F.logsigmoid(-logits)
        if s.r == 0:
            # pure-GLA branch, Train.py:201-223
            Y_I, S = chunk_gla_core(Q, K, V, log_gamma, 0, s.chunk_size,
                                    log_alpha=self._log_alpha(), dtype=self.dtype, mode=self.gla_mode)
            var = (Y_I * Y_I).mean(-1, keepdim=True)
            Y_I = Y_I * torch.rsqrt(var + FP32_EPS) * self.p['gla_scale'].reshape(1, s.num_heads, 1, s.d_head)
            out = self._out(self._act(Y_I))
            return (out, None, S) if return_state else out
        Q_O, K_O = Q[..., :s.r], K[..., :s.r]
        if s.use_rope:
            cos, sin = rope_cos_sin(s.r, N, s.rope_base, self.dtype)
            Q_O, K_O = apply_rope(Q_O, cos, sin), apply_rope(K_O, cos, sin)
            Q_O, K_O = self._act(Q_O), self._act(K_O)
        sm_scale = (s.d_head / s.r) ** 0.5 * s.attention_scale
        Y_O = outlier_attention_core(Q_O, K_O, V, s.r, sm_scale,
                                     torch.ones(B, s.num_heads, N, dtype=self.dtype), dtype=self.dtype)
        Y_I, S = chunk_gla_core(Q, K, V, log_gamma, s.r, s.chunk_size,
                                log_alpha=self._log_alpha(), dtype=self.dtype, mode=self.gla_mode)
        var = (Y_I * Y_I).mean(-1, keepdim=True)
        Y_I = Y_I * torch.rsqrt(var + self.prefill_eps) * self.p['gla_scale'].reshape(1, s.num_heads, 1, s.d_head)
        m = mix[..., None]
        Y = Y_I + m * (Y_O - Y_I)          # torch.lerp(Y_I, Y_O, mix_g), Train.py:294
        out = self._out(Y)
        if return_state:
            return out, (K_O.contiguous(), V.contiguous()), S
        return out

    # -- decode: Train.forward_step (:382-438) ------------------------------
    def forward_step(self, x, cache_O=None, state_I=None):
        """Hybrid branch of Train.forward_step with the inference-module state
        layout: ``state_I`` is ``[B,H,j,D]`` (the Train module keeps
        ``[B,H,D,D]`` with zero rows ``[j:]``, Train.py:411-423).  Returns
        ``(out, (K_cache, V_cache), state_new)``."""
        s = self.s
        B, N, _ = x.shape
        assert N == 1
        Q, K, V = self._proj(x)
        logits, mix = self.gates(Q, K)
        if state_I is None:
            state_I = torch.zeros(B, s.num_heads, s.j, s.d_head, dtype=self.dtype)
        if s.r == 0:
            # pure-GLA branch, Train.py:340-362: no outlier cache, no blend
            zero = torch.zeros(B, s.num_heads, 1, dtype=self.dtype)
            y, S_new = decode_core(Q, K, V, None, None, state_I, F.logsigmoid(-logits), zero,
                                   self.p['gla_scale'].reshape(s.num_heads, s.d_head), 0, 0, 1.0,
                                   log_alpha=self._log_alpha(), eps=FP32_EPS, dtype=self.dtype)
            return self._out(self._act(y)), None, S_new
        pos = 0 if cache_O is None else cache_O[0].shape[2]
        Q_O, K_O = Q[..., :s.r], K[..., :s.r]
        if s.use_rope:
            cos, sin = rope_cos_sin(s.r, pos + 1, s.rope_base, self.dtype)
            Q_O, K_O = apply_rope(Q_O, cos[-1:], sin[-1:]), apply_rope(K_O, cos[-1:], sin[-1:])
            Q_O, K_O = self._act(Q_O), self._act(K_O)
        if cache_O is None:
            Kc, Vc = K_O, V
        else:
            Kc = torch.cat([cache_O[0].to(self.dtype), K_O], dim=2)
            Vc = torch.cat([cache_O[1].to(self.dtype), V], dim=2)
        q = torch.cat([Q_O, Q[..., s.r:]], dim=-1)
        y, S_new = decode_core(q, K, V, Kc, Vc, state_I, F.logsigmoid(-logits), mix,
                               self.p['gla_scale'].reshape(s.num_heads, s.d_head),
                               s.r, Kc.shape[2], (s.d_head / s.r) ** 0.5,
                               log_alpha=self._log_alpha(), eps=FP32_EPS, dtype=self.dtype)
        return self._out(y), (Kc, Vc), S_new
