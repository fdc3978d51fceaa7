"""Drop-in HOFA layer: ``HybridOutlierFactorizedAttention``.

Same constructor, parameter/buffer names, ``forward(x, return_state)`` and
``forward_step(x, cache_O, state_I, cache_seq_len)`` as the reference
inference module (src/HybridOutlierFactorizedAttention.py:11-422 of
LotanGutman/OutlierNeuronAttention), same cache layouts:

* outlier KV cache ``(K_O [B,H,L,r] RoPE-rotated, V [B,H,L,d_h])``;
* GLA state ping-pong ``(state_in, state_out)``, each ``[B,H,j,d_h]`` float32,
  returned swapped by ``forward_step``.

The hybrid path runs on hand-written sm_100a kernels: ``hofa_prep_fwd``
(gates, logsigmoid, RoPE, cache export/append), ``hofa_prefill_gla_fwd``,
``hofa_prefill_outlier_fwd`` and ``hofa_decode_fwd``.  The projections are
cuBLAS GEMMs (``nn.Linear``).  The ablation branches that contain no HOFA
kernel in the reference either (``r == d_head``: plain SDPA; width split:
SDPA heads + GLA heads) follow the reference's PyTorch code, with the GLA
heads of the width split on the native GLA kernel.

RMSNorm epsilon: float32 machine epsilon for prefill and decode by default,
as in the reference's decode kernel and its training layer
(src/HybridOutlierFactorizedAttentionTrain.py:71, nn.RMSNorm with eps=None).
The reference's inference layer hard-codes 1e-5 in its hybrid prefill
(src/HybridOutlierFactorizedAttention.py:203-206 -> src/chunk_gla_inlier.py:234)
while its decode uses float32 epsilon; where the GLA outputs are small (early
tokens, small projections) the two epsilons give visibly different normalised
outputs.  ``layer.hybrid_prefill_eps = 1e-5`` reproduces the inference
layer's prefill.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .chunk_gla_inlier import chunk_gla_inlier_fwd, gla_forward
from .config import ModelConfig
from .exact_attention import exact_attention_triton
from .hofa_decode import fused_hofa_decode, fused_hofa_decode_step
from .modules import RotaryEmbedding, apply_rotary_pos_emb
from .prep import prep

FP32_EPS = float(torch.finfo(torch.float32).eps)


class HybridOutlierFactorizedAttention(nn.Module):
    def __init__(self, model_cfg: ModelConfig):
        super().__init__()
        self.d_model = model_cfg.d_model
        self.num_heads = model_cfg.num_heads
        self.d_head = model_cfg.d_head
        self.r = model_cfg.r
        self.j = self.d_head - self.r
        self.chunk_size = model_cfg.chunk_size

        self.gate_proj = nn.Linear(2 * self.d_head, self.num_heads, bias=True)
        nn.init.constant_(self.gate_proj.bias, -1.0)
        nn.init.zeros_(self.gate_proj.weight)

        self.forced_mha_heads = getattr(model_cfg, "mha_heads_for_width_split", 0)
        self.fixed_blend_weight = getattr(model_cfg, "fixed_blend_weight", False)
        if not self.fixed_blend_weight and self.forced_mha_heads == 0:
            self.mix_proj = nn.Linear(2 * self.d_head, self.num_heads, bias=True)
            nn.init.zeros_(self.mix_proj.weight)
            nn.init.constant_(self.mix_proj.bias, model_cfg.mix_gate_bias_init)
        elif self.fixed_blend_weight and self.forced_mha_heads == 0:
            self.fixed_mix = nn.Parameter(torch.zeros(1, self.num_heads, 1, 1))

        self.learnable_alpha = getattr(model_cfg, "learnable_alpha", False)
        if self.learnable_alpha:
            n_dec = self.d_head if self.forced_mha_heads > 0 else (self.d_head if self.r == 0 else self.j)
            self.log_alpha = nn.Parameter(torch.zeros(1, self.num_heads, 1, n_dec))
            self.log_alpha._is_alpha = True

        self.W_q = nn.Linear(self.d_model, self.d_model, bias=False)
        self.W_k = nn.Linear(self.d_model, self.d_model, bias=False)
        self.W_v = nn.Linear(self.d_model, self.d_model, bias=False)
        self.out_proj = nn.Linear(self.d_model, self.d_model, bias=False)

        if (self.r > 0 or self.forced_mha_heads > 0) and model_cfg.use_rope:
            self.rotary_emb = RotaryEmbedding(dim=self.r if self.r > 0 else self.d_head, base=model_cfg.rope_base)

        self.inlier_norm = nn.RMSNorm(self.d_head, elementwise_affine=False)
        self.gla_scale = nn.Parameter(torch.ones(1, self.num_heads, 1, self.d_head))
        # RMSNorm epsilon of the hybrid prefill (see the module docstring); not a parameter or buffer
        self.hybrid_prefill_eps = FP32_EPS

    # ------------------------------------------------------------------ helpers
    def _qkv_weight(self):
        """[W_q / d_h^(1/4); W_k / d_h^(1/4); W_v] as one [3*H*d_h, d_model]
        weight (the reference's scaling, :100-104, folded in fp32), rebuilt
        whenever one of the three weights is replaced or modified in place."""
        ws = (self.W_q.weight, self.W_k.weight, self.W_v.weight)
        key = tuple((w.data_ptr(), w._version, w.dtype, w.device) for w in ws)
        if getattr(self, "_qkv_key", None) != key:
            sf = self.d_head ** 0.25
            self._qkv_w = torch.cat([(ws[0].float() / sf).to(ws[0].dtype), (ws[1].float() / sf).to(ws[1].dtype),
                                     ws[2]], dim=0).detach()
            self._qkv_key = key
        return self._qkv_w

    def _project(self, x):
        """Q, K, V [B,H,N,d_h] as strided views of one projection GEMM."""
        B, N, _ = x.shape
        qkv = F.linear(x, self._qkv_weight()).view(B, N, 3, self.num_heads, self.d_head)
        return qkv[:, :, 0].transpose(1, 2), qkv[:, :, 1].transpose(1, 2), qkv[:, :, 2].transpose(1, 2)

    def _gate_kwargs(self):
        kw = dict(gate_w=self.gate_proj.weight, gate_b=self.gate_proj.bias)
        if hasattr(self, "mix_proj"):
            kw.update(mix_w=self.mix_proj.weight, mix_b=self.mix_proj.bias)
        elif hasattr(self, "fixed_mix"):
            kw.update(fixed_mix=self.fixed_mix.view(self.num_heads))
        return kw

    def _rope_tables(self, n_positions: int):
        if not hasattr(self, "rotary_emb"):
            return None, None
        self.rotary_emb(n_positions)  # grows the tables when needed
        return self.rotary_emb.cos_cached, self.rotary_emb.sin_cached

    def _prep(self, Q, K, V, N, pos0, mix_out=True, cache_k=None, cache_v=None):
        B = Q.shape[0]
        log_gamma = torch.empty(B, self.num_heads, N, dtype=torch.float32, device=Q.device)
        mix = torch.empty(B, self.num_heads, N, dtype=Q.dtype, device=Q.device) if mix_out else None
        cos, sin = self._rope_tables(pos0 + N) if self.r > 0 else (None, None)
        prep(Q, K, V, log_gamma=log_gamma, mix_out=mix, cos=cos, sin=sin, R=self.r,
             pos0=pos0, cache_k=cache_k, cache_v=cache_v, use_rope=cos is not None, **self._gate_kwargs())
        return log_gamma, mix

    def _out(self, Y, B, N, dtype_in):
        return self.out_proj(Y.transpose(1, 2).reshape(B, N, self.d_model)).to(dtype_in)

    # ------------------------------------------------------------------ prefill
    def forward(self, x, return_state=False):
        B, N, D = x.shape
        dtype_in = x.dtype
        Q, K, V = self._project(x)

        if self.forced_mha_heads > 0:
            return self._forward_width_split(Q, K, V, B, N, dtype_in, return_state)

        if self.r == 0:
            log_gamma, _ = self._prep(Q, K, V, N, 0, mix_out=False)
            zero_mix = torch.zeros(B, self.num_heads, N, dtype=Q.dtype, device=Q.device)
            state = (torch.empty(B, self.num_heads, self.j, self.d_head, dtype=torch.float32, device=Q.device)
                     if return_state else None)
            Y = gla_forward(Q, K, V, log_gamma, 0, log_alpha=getattr(self, "log_alpha", None) if self.learnable_alpha else None,
                            mix_g=zero_mix, gla_scale=self.gla_scale, state_out=state, eps=FP32_EPS)
            Y_out = self._out(Y, B, N, dtype_in)
            if return_state:
                return Y_out, None, (state, torch.empty_like(state))
            return Y_out

        if self.r == self.d_head:
            if hasattr(self, "rotary_emb"):
                cos, sin = self.rotary_emb(N)
                Q, K = apply_rotary_pos_emb(Q, K, cos, sin)
            Y = F.scaled_dot_product_attention(Q, K, V, is_causal=True, scale=1.0)
            Y_out = self._out(Y, B, N, dtype_in)
            if return_state:
                return Y_out, (K.contiguous(), V.contiguous()), None
            return Y_out

        # ----- hybrid: prep -> GLA (writes Y) -> outlier attention (adds into Y)
        K_cache = V_cache = None
        if return_state:
            K_cache = torch.empty(B, self.num_heads, N, self.r, dtype=K.dtype, device=K.device)
            V_cache = torch.empty(B, self.num_heads, N, self.d_head, dtype=V.dtype, device=V.device)
        log_gamma, mix = self._prep(Q, K, V, N, 0, cache_k=K_cache, cache_v=V_cache)
        state = (torch.empty(B, self.num_heads, self.j, self.d_head, dtype=torch.float32, device=Q.device)
                 if return_state else None)
        Y = gla_forward(Q, K, V, log_gamma, self.r,
                        log_alpha=self.log_alpha if self.learnable_alpha else None,
                        mix_g=mix, gla_scale=self.gla_scale, state_out=state, eps=self.hybrid_prefill_eps)
        sm_scale = (self.d_head / self.r) ** 0.5
        exact_attention_triton(Q, K, V, self.r, sm_scale, mix, out=Y)
        Y_out = self._out(Y, B, N, dtype_in)
        if return_state:
            return Y_out, (K_cache, V_cache), (state, torch.empty_like(state))
        return Y_out

    def _forward_width_split(self, Q, K, V, B, N, dtype_in, return_state):
        """Width-split ablation (reference :106-143): SDPA heads + GLA heads."""
        fm, H = self.forced_mha_heads, self.num_heads
        Q_mha, Q_gla = Q.split([fm, H - fm], dim=1)
        K_mha, K_gla = K.split([fm, H - fm], dim=1)
        V_mha, V_gla = V.split([fm, H - fm], dim=1)
        if hasattr(self, "rotary_emb"):
            cos, sin = self.rotary_emb(N)
            Q_mha, K_mha = apply_rotary_pos_emb(Q_mha, K_mha, cos, sin)
        Y_mha = F.scaled_dot_product_attention(Q_mha, K_mha, V_mha, is_causal=True, scale=1.0)
        W_g_q, W_g_k = self.gate_proj.weight.chunk(2, dim=1)
        b_g = self.gate_proj.bias[fm:].view(1, -1, 1).to(dtype_in)
        gate_logits = (torch.einsum("bhnf,hf->bhn", Q_gla, W_g_q[fm:]) +
                       torch.einsum("bhnf,hf->bhn", K_gla, W_g_k[fm:]) + b_g)
        log_gamma = F.logsigmoid(-gate_logits)
        Y_gla, states_out = chunk_gla_inlier_fwd(Q_gla, K_gla, V_gla, log_gamma, 0, self.chunk_size)
        Y_gla = (self.inlier_norm(Y_gla.float()) * self.gla_scale[:, fm:]).to(Y_gla.dtype)
        Y_out = self._out(torch.cat([Y_mha, Y_gla], dim=1), B, N, dtype_in)
        if return_state:
            state_I = states_out[:, :, :self.d_head, :self.d_head]
            return Y_out, (K_mha.contiguous(), V_mha.contiguous()), (state_I, torch.empty_like(state_I))
        return Y_out

    # ------------------------------------------------------------------ decode
    def forward_step(self, x, cache_O=None, state_I=None, cache_seq_len=None):
        """Single-step autoregressive decoding (reference :223-422)."""
        B, N, D = x.shape
        assert N == 1, "forward_step expects a single token (N=1)"
        dtype_in = x.dtype
        Q, K, V = self._project(x)

        if self.forced_mha_heads > 0:
            return self._step_width_split(Q, K, V, B, N, D, dtype_in, cache_O, state_I, cache_seq_len)

        if self.r == 0:
            log_gamma, _ = self._prep(Q, K, V, 1, 0, mix_out=False)
            if isinstance(state_I, tuple):
                state_in, state_out = state_I
            else:
                state_in, state_out = state_I, None
            if state_in is None:
                state_in = torch.zeros(B, self.num_heads, self.j, self.d_head, device=x.device, dtype=torch.float32)
            if state_out is None or state_out.shape != state_in.shape or state_out.data_ptr() == state_in.data_ptr():
                state_out = torch.empty_like(state_in)
            zero_mix = torch.zeros(B, self.num_heads, 1, dtype=Q.dtype, device=Q.device)
            Y = fused_hofa_decode(Q, K, V, None, None, state_in, state_out, log_gamma, zero_mix,
                                  self.gla_scale.view(self.num_heads, self.d_head), 0, 1, 1.0,
                                  log_alpha=self.log_alpha if self.learnable_alpha else None)
            return self._out(Y, B, N, dtype_in), None, (state_out, state_in)

        if self.r == self.d_head:
            return self._step_full_attention(Q, K, V, B, N, dtype_in, cache_O, cache_seq_len)

        # ----- hybrid step
        seq_idx = cache_seq_len if cache_seq_len is not None else (cache_O[0].shape[2] if cache_O is not None else 0)
        if state_I is None:
            state_I = (torch.zeros(B, self.num_heads, self.j, self.d_head, device=x.device, dtype=torch.float32),
                       torch.empty(B, self.num_heads, self.j, self.d_head, device=x.device, dtype=torch.float32))
        if torch.is_tensor(cache_seq_len):
            return self._step_device_position(Q, K, V, B, N, dtype_in, cache_O, state_I, cache_seq_len)
        if cache_O is not None and cache_seq_len is not None and cache_O[0].shape[2] > cache_seq_len:
            # pre-allocated cache (the serving path): gates, RoPE at row
            # cache_seq_len, the cache append and the decode core in one launch
            state_in, state_out = state_I
            assert state_in.dtype == torch.float32, f"Expected state_in to be float32, got {state_in.dtype}"
            assert state_in.is_contiguous(), "Expected state_in to be contiguous"
            cos, sin = self._rope_tables(seq_idx + 1)
            Y, _, _ = fused_hofa_decode_step(
                Q, K, V, cache_O[0], cache_O[1], state_in, state_out,
                self.gla_scale.view(self.num_heads, self.d_head), self.r, cache_seq_len + 1,
                (self.d_head / self.r) ** 0.5, cos=cos, sin=sin,
                log_alpha=self.log_alpha if self.learnable_alpha else None, **self._gate_kwargs())
            return self._out(Y, B, N, dtype_in), cache_O, (state_out, state_in)
        if cache_O is None:
            log_gamma, mix = self._prep(Q, K, V, 1, seq_idx)
            K_past, V_past = K[..., :self.r], V
            cache_O_new = (K_past, V_past)
            cache_seq_len = 0
        else:
            log_gamma, mix = self._prep(Q, K, V, 1, seq_idx)
            K_past = torch.cat([cache_O[0], K[..., :self.r]], dim=2)
            V_past = torch.cat([cache_O[1], V], dim=2)
            cache_O_new = (K_past, V_past)
            cache_seq_len = K_past.shape[2] - 1

        state_in, state_out = state_I
        assert state_in.dtype == torch.float32, f"Expected state_in to be float32, got {state_in.dtype}"
        assert state_in.is_contiguous(), "Expected state_in to be contiguous"

        sm_scale = (self.d_head / self.r) ** 0.5
        Y = fused_hofa_decode(Q, K, V, K_past, V_past, state_in, state_out, log_gamma, mix,
                              self.gla_scale.view(self.num_heads, self.d_head), self.r, cache_seq_len + 1,
                              sm_scale, log_alpha=self.log_alpha if self.learnable_alpha else None)
        return self._out(Y, B, N, dtype_in), cache_O_new, (state_out, state_in)

    def _step_device_position(self, Q, K, V, B, N, dtype_in, cache_O, state_I, cache_seq_len):
        """Decode step whose position lives on the device: ``cache_seq_len`` is
        an int32 CUDA scalar holding the rows already in the pre-allocated
        ``cache_O``, so a decode loop can be captured once in a CUDA graph and
        replayed with the position advanced on the device (no host value, no
        synchronisation).  The RoPE tables are sized to the cache's capacity;
        a position outside the cache is clamped and flagged in the decode
        workspace's status word."""
        if cache_O is None:
            raise ValueError("a device-side cache_seq_len needs a pre-allocated cache_O")
        if cache_seq_len.dtype != torch.int32 or cache_seq_len.numel() != 1 or not cache_seq_len.is_cuda:
            raise ValueError("a device-side cache_seq_len is a one-element int32 CUDA tensor")
        state_in, state_out = state_I
        assert state_in.dtype == torch.float32, f"Expected state_in to be float32, got {state_in.dtype}"
        assert state_in.is_contiguous(), "Expected state_in to be contiguous"
        L = cache_O[0].shape[2]
        cos, sin = self._rope_tables(L)
        buf = getattr(self, "_seq_len_dev", None)
        if buf is None or buf.device != cache_seq_len.device:
            buf = torch.empty(1, dtype=torch.int32, device=cache_seq_len.device)
            self._seq_len_dev = buf
        torch.add(cache_seq_len.view(1), 1, out=buf)  # rows attended: the cache's plus the new one
        Y, _, _ = fused_hofa_decode_step(
            Q, K, V, cache_O[0], cache_O[1], state_in, state_out,
            self.gla_scale.view(self.num_heads, self.d_head), self.r, L, (self.d_head / self.r) ** 0.5,
            cos=cos, sin=sin, seq_len_dev=buf,
            log_alpha=self.log_alpha if self.learnable_alpha else None, **self._gate_kwargs())
        return self._out(Y, B, N, dtype_in), cache_O, (state_out, state_in)

    def _append(self, cache_O, K_new, V_new, cache_seq_len):
        if cache_O is None:
            return K_new, V_new, (K_new, V_new)
        if cache_seq_len is not None and cache_O[0].shape[2] > cache_seq_len:
            cache_O[0][:, :, cache_seq_len:cache_seq_len + 1, :] = K_new
            cache_O[1][:, :, cache_seq_len:cache_seq_len + 1, :] = V_new
            return cache_O[0][:, :, :cache_seq_len + 1, :], cache_O[1][:, :, :cache_seq_len + 1, :], cache_O
        K_past = torch.cat([cache_O[0], K_new], dim=2)
        V_past = torch.cat([cache_O[1], V_new], dim=2)
        return K_past, V_past, (K_past, V_past)

    def _rope_at(self, Q, K, cache_O, cache_seq_len):
        seq_idx = cache_seq_len if cache_seq_len is not None else (cache_O[0].shape[2] if cache_O is not None else 0)
        cos, sin = self.rotary_emb(seq_idx + 1)
        return apply_rotary_pos_emb(Q, K, cos[-1:, :], sin[-1:, :])

    def _step_full_attention(self, Q, K, V, B, N, dtype_in, cache_O, cache_seq_len):
        """r == d_head (reference :333-356): plain attention over the cache."""
        if hasattr(self, "rotary_emb"):
            Q, K = self._rope_at(Q, K, cache_O, cache_seq_len)
        if cache_O is not None and cache_seq_len is not None and cache_O[0].shape[2] > cache_seq_len:
            K_past, V_past, _ = self._append(cache_O, K, V, cache_seq_len)
            cache_new = cache_O
        else:
            K_past, V_past, cache_new = self._append(cache_O, K, V, cache_seq_len)
        Y = F.scaled_dot_product_attention(Q, K_past, V_past, is_causal=False, scale=1.0)
        return self._out(Y, B, N, dtype_in), cache_new, None

    def _step_width_split(self, Q, K, V, B, N, D, dtype_in, cache_O, state_I, cache_seq_len):
        """Width-split ablation decode (reference :234-296)."""
        fm, H = self.forced_mha_heads, self.num_heads
        Hg = H - fm
        Q_mha, Q_gla = Q.split([fm, Hg], dim=1)
        K_mha, K_gla = K.split([fm, Hg], dim=1)
        V_mha, V_gla = V.split([fm, Hg], dim=1)
        if hasattr(self, "rotary_emb"):
            Q_mha, K_mha = self._rope_at(Q_mha, K_mha, cache_O, cache_seq_len)
        K_past, V_past, cache_new = self._append(cache_O, K_mha, V_mha, cache_seq_len)
        Y_mha = F.scaled_dot_product_attention(Q_mha, K_past, V_past, is_causal=False, scale=1.0)
        W_g_q, W_g_k = self.gate_proj.weight.chunk(2, dim=1)
        b_g = self.gate_proj.bias[fm:].view(1, -1, 1).to(dtype_in)
        gate_logits = (torch.einsum("bhnf,hf->bhn", Q_gla, W_g_q[fm:]) +
                       torch.einsum("bhnf,hf->bhn", K_gla, W_g_k[fm:]) + b_g)
        gamma = torch.sigmoid(-gate_logits).view(B, Hg, 1, 1)
        S = (torch.zeros(B, Hg, self.d_head, self.d_head, device=Q.device, dtype=torch.float32)
             if state_I is None else state_I[0])
        k_s = K_gla.squeeze(2).float().unsqueeze(-1)
        v_s = V_gla.squeeze(2).float().unsqueeze(-2)
        S_new = S * gamma + k_s @ v_s
        Y_gla = (Q_gla.squeeze(2).float().unsqueeze(-2) @ S_new).reshape(B, Hg, 1, self.d_head)
        Y_gla = (self.inlier_norm(Y_gla.float()) * self.gla_scale[:, fm:]).to(dtype_in)
        Y_out = self._out(torch.cat([Y_mha, Y_gla], dim=1), B, N, dtype_in)
        return Y_out, cache_new, (S_new, torch.empty_like(S_new))
