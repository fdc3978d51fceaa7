"""A decoder LM around the drop-in HOFA layer, and a graph-replayed decode engine.

The LM is the harness the decode benchmark of a full model needs: token
embedding, ``num_layers`` pre-norm blocks of (RMSNorm, the drop-in
``HybridOutlierFactorizedAttention``, RMSNorm, SwiGLU MLP), a final RMSNorm
and a language-model head tied to the embedding.  At the 350M shape (24
layers, d_model 1024, 16 heads of 64, r = 16, MLP 4096, vocabulary 32000) it
holds 435.6M parameters.  The attention of every layer runs on this
library's kernels; in decode steps of up to 8 sequences the projections and
the MLP run on its small-batch linear kernel (``hofa_lm_linear_fwd``, with the
RMSNorm, the SwiGLU product and the residual add folded in), otherwise (and in
the prefill) as cuBLAS GEMMs.

``DecodeEngine`` replaces the per-token host loop of the reference's
generation (src/inference.py:174-239, one ``.item()`` per token and the
position as a host integer) with a CUDA graph of two decode steps: the
position lives in a device int32 that every layer's ``forward_step`` reads
(the layer's device-position path: RoPE row, cache row and attended length
come from it) and that the graph advances; the next token is sampled inside
the graph (greedy, or temperature with top-k through the Gumbel-max trick on
the device generator), written into a device token buffer and fed to the next
step.  Two steps per graph because each layer's GLA state ping-pongs between
two buffers.  Nothing is synchronised until the caller reads the tokens.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _capi
from ._capi import LinearArgs, flat, tview
from .config import ModelConfig
from .hofa_decode import fused_hofa_decode_step
from .layer import HybridOutlierFactorizedAttention


def lm_linear(x: torch.Tensor, weight: torch.Tensor, y: torch.Tensor, *, norm_w: Optional[torch.Tensor] = None,
              residual: Optional[torch.Tensor] = None, mode: int = 0, eps: float = 1e-6) -> torch.Tensor:
    """``y = (residual +) transform(x) @ weight.T`` for decode-sized batches
    (``hofa_lm_linear_fwd``): x [M, K] (or [M, 2K] = [gate | up] with mode 2),
    weight [N, K], y [M, N], M <= 8, bf16/f16.  mode 0: x; 1: RMSNorm(x) *
    norm_w; 2: silu(gate) * up.  ``residual`` may be ``y`` itself."""
    vals = flat(tview(x), tview(weight), tview(norm_w), tview(residual), tview(y), int(mode), float(eps))
    _capi.call("hofa_lm_linear_fwd", LinearArgs, vals, _capi.stream_handle(x.device))
    return y


@dataclass
class LMConfig:
    vocab_size: int = 32000
    d_model: int = 1024
    num_heads: int = 16
    num_layers: int = 24
    r: int = 16
    d_mlp: int = 4096
    chunk_size: int = 64
    norm_eps: float = 1e-6
    init_std: float = 0.02

    def layer_config(self) -> ModelConfig:
        return ModelConfig(d_model=self.d_model, num_heads=self.num_heads, num_layers=self.num_layers, r=self.r,
                           chunk_size=self.chunk_size)


class SwiGLU(nn.Module):
    def __init__(self, d_model: int, d_mlp: int):
        super().__init__()
        self.gate_up = nn.Linear(d_model, 2 * d_mlp, bias=False)
        self.down = nn.Linear(d_mlp, d_model, bias=False)

    def forward(self, x):
        g, u = self.gate_up(x).chunk(2, dim=-1)
        return self.down(F.silu(g) * u)


class Block(nn.Module):
    def __init__(self, cfg: LMConfig):
        super().__init__()
        self.attn_norm = nn.RMSNorm(cfg.d_model, eps=cfg.norm_eps)
        self.attn = HybridOutlierFactorizedAttention(cfg.layer_config())
        self.mlp_norm = nn.RMSNorm(cfg.d_model, eps=cfg.norm_eps)
        self.mlp = SwiGLU(cfg.d_model, cfg.d_mlp)


class HofaLM(nn.Module):
    def __init__(self, cfg: LMConfig):
        super().__init__()
        self.cfg = cfg
        self.embed = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.blocks = nn.ModuleList([Block(cfg) for _ in range(cfg.num_layers)])
        self.norm = nn.RMSNorm(cfg.d_model, eps=cfg.norm_eps)
        self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self):
        std = self.cfg.init_std
        for name, p in self.named_parameters():
            if name.endswith("weight") and p.dim() == 2 and "gate_proj" not in name and "mix_proj" not in name:
                p.normal_(0.0, std)
        for b in self.blocks:   # gates vary per token (the layer's own init keeps them constant)
            b.attn.gate_proj.weight.normal_(0.0, std)
            if hasattr(b.attn, "mix_proj"):
                b.attn.mix_proj.weight.normal_(0.0, std)

    def num_parameters(self) -> int:
        return sum(p.numel() for p in self.parameters())

    def logits(self, x):
        return F.linear(self.norm(x), self.embed.weight)

    @torch.no_grad()
    def prefill(self, idx: torch.Tensor, capacity: int, batch_chunk: Optional[int] = None):
        """Runs the prompt ``idx`` [B, T] through every layer's prefill and
        returns (logits of the last token [B, vocab], caches, states): per
        layer a pre-allocated outlier cache ``(K [B,H,capacity,r], V
        [B,H,capacity,d_head])`` holding rows [0, T) and a GLA state pair
        ``(state, spare)``.  ``batch_chunk`` runs the prompt that many
        sequences at a time (bounds the activation memory)."""
        B, T = idx.shape
        cfg = self.cfg
        d_head = cfg.d_model // cfg.num_heads
        dev = idx.device
        dt = self.embed.weight.dtype
        caches = [(torch.zeros(B, cfg.num_heads, capacity, cfg.r, device=dev, dtype=dt),
                   torch.zeros(B, cfg.num_heads, capacity, d_head, device=dev, dtype=dt)) for _ in self.blocks]
        states = [(torch.empty(B, cfg.num_heads, d_head - cfg.r, d_head, device=dev, dtype=torch.float32),
                   torch.empty(B, cfg.num_heads, d_head - cfg.r, d_head, device=dev, dtype=torch.float32))
                  for _ in self.blocks]
        step = batch_chunk or B
        last = []
        for b0 in range(0, B, step):
            b1 = min(B, b0 + step)
            x = self.embed(idx[b0:b1])
            for blk, (ck, cv), (s0, _) in zip(self.blocks, caches, states):
                y, (k, v), (st, _) = blk.attn(blk.attn_norm(x), return_state=True)
                ck[b0:b1, :, :T].copy_(k)
                cv[b0:b1, :, :T].copy_(v)
                s0[b0:b1].copy_(st)
                x = x + y
                x = x + blk.mlp(blk.mlp_norm(x))
            last.append(self.logits(x[:, -1]))
        return torch.cat(last, 0), caches, states

    def fused_step_ok(self, B: int) -> bool:
        """Whether a decode step of B sequences runs on the fused small-batch path."""
        return B <= 8 and self.embed.weight.dtype in (torch.bfloat16, torch.float16) and self.embed.weight.is_cuda

    def step(self, tok: torch.Tensor, caches, states, pos_dev: torch.Tensor, flip: bool, fused: Optional[bool] = None):
        """One decode step for tokens ``tok`` [B, 1] at the device position
        ``pos_dev`` (int32 [1]: rows already in the caches).  ``flip`` selects
        the direction of the GLA state ping-pong.  Returns logits [B, vocab].

        Up to 8 sequences in bf16/f16 (``fused``, the default there) a layer is
        five launches: RMSNorm + QKV projection, the layer's one-launch decode
        step (gates, RoPE, cache append, attention core), out-projection +
        residual, RMSNorm + gate/up projection, SwiGLU + down-projection +
        residual (``hofa_lm_linear_fwd`` streams each weight once).  Otherwise
        the modules run as written (the layer's ``forward_step``, nn.Linear)."""
        B = tok.shape[0]
        if fused is None:
            fused = self.fused_step_ok(B)
        if not fused:
            x = self.embed(tok)
            for blk, cache, (s0, s1) in zip(self.blocks, caches, states):
                st = (s1, s0) if flip else (s0, s1)
                y, _, _ = blk.attn.forward_step(blk.attn_norm(x), cache, st, cache_seq_len=pos_dev)
                x = x + y
                x = x + blk.mlp(blk.mlp_norm(x))
            return self.logits(x[:, -1])
        cfg = self.cfg
        H, dh = cfg.num_heads, cfg.d_model // cfg.num_heads
        x = self.embed(tok).view(B, cfg.d_model)
        seq_len = pos_dev + 1                        # rows attended: the cached ones and the new one
        qkv = torch.empty(B, 3 * cfg.d_model, device=x.device, dtype=x.dtype)
        gu = torch.empty(B, 2 * cfg.d_mlp, device=x.device, dtype=x.dtype)
        for blk, (ck, cv), (s0, s1) in zip(self.blocks, caches, states):
            at = blk.attn
            s_in, s_out = (s1, s0) if flip else (s0, s1)
            lm_linear(x, at._qkv_weight(), qkv, norm_w=blk.attn_norm.weight, mode=1, eps=blk.attn_norm.eps)
            q, k, v = (t.transpose(1, 2) for t in qkv.view(B, 1, 3, H, dh).unbind(2))
            cos, sin = at._rope_tables(ck.shape[2])
            y, _, _ = fused_hofa_decode_step(
                q, k, v, ck, cv, s_in, s_out, at.gla_scale.view(H, dh), at.r, ck.shape[2], (dh / at.r) ** 0.5,
                cos=cos, sin=sin, seq_len_dev=seq_len, log_alpha=at.log_alpha if at.learnable_alpha else None,
                **at._gate_kwargs())
            lm_linear(y.reshape(B, cfg.d_model), at.out_proj.weight, x, residual=x)
            lm_linear(x, blk.mlp.gate_up.weight, gu, norm_w=blk.mlp_norm.weight, mode=1, eps=blk.mlp_norm.eps)
            lm_linear(gu, blk.mlp.down.weight, x, residual=x, mode=2)
        logits = torch.empty(B, cfg.vocab_size, device=x.device, dtype=x.dtype)
        return lm_linear(x, self.embed.weight, logits, norm_w=self.norm.weight, mode=1, eps=self.norm.eps)


def sample_tokens(logits: torch.Tensor, temperature: float, top_k: int) -> torch.Tensor:
    """Next tokens [B] from logits [B, V] on the device, without a host sync:
    greedy when ``temperature`` is 0, else Gumbel-max over the top-k logits
    divided by the temperature (the same distribution as softmax sampling
    of the top-k)."""
    if temperature <= 0:
        return logits.argmax(dim=-1)
    vals, idx = logits.float().topk(top_k, dim=-1)
    u = torch.rand_like(vals).clamp_(1e-20, 1.0)
    choice = (vals / temperature - torch.log(-torch.log(u))).argmax(dim=-1, keepdim=True)
    return idx.gather(-1, choice).squeeze(-1)


class DecodeEngine:
    """Graph-replayed generation for ``HofaLM`` (see the module docstring).

    ``first_logits`` are the prefill's last-token logits; ``prompt_len`` the
    rows already in the caches.  ``generate(n)`` (n even) samples the first
    token from ``first_logits`` and then replays the two-step graph n/2
    times (n decode steps); returns the tokens [B, n + 1] (the first one and
    the n sampled by the steps; a device tensor, nothing synchronised).  The
    caches must hold ``prompt_len + n`` rows.  Every call starts again from
    the prompt (the GLA states are restored, the cache rows overwritten)."""

    def __init__(self, model: HofaLM, caches, states, first_logits: torch.Tensor, prompt_len: int,
                 temperature: float = 0.0, top_k: int = 50):
        self.model, self.caches, self.states = model, caches, states
        self.B = first_logits.shape[0]
        self.dev = first_logits.device
        self.prompt_len = prompt_len
        self.temperature, self.top_k = temperature, top_k
        self.first_logits = first_logits
        self.capacity = caches[0][0].shape[2]
        self.pos = torch.full((1,), prompt_len, dtype=torch.int32, device=self.dev)
        self.tok = torch.zeros(self.B, 1, dtype=torch.long, device=self.dev)
        self.count = torch.zeros(1, dtype=torch.long, device=self.dev)
        self.out: Optional[torch.Tensor] = None
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.stream = torch.cuda.Stream(self.dev)

    def _two_steps(self):
        for flip in (False, True):
            logits = self.model.step(self.tok, self.caches, self.states, self.pos, flip)
            nxt = sample_tokens(logits, self.temperature, self.top_k)
            self.tok.copy_(nxt[:, None])
            self.out.scatter_(1, self.count.expand(self.B, 1), self.tok)
            self.pos.add_(1)
            self.count.add_(1)

    @torch.no_grad()
    def capture(self, max_tokens: int):
        """Warms every layer up (workspaces, RoPE tables) and captures the
        two-step graph.  The warm-up steps run at the prompt's position and
        are undone (their cache rows are overwritten by the real steps; the
        states are restored)."""
        if self.prompt_len + max_tokens > self.capacity:
            raise ValueError(f"caches hold {self.capacity} rows, need {self.prompt_len + max_tokens}")
        self.out = torch.zeros(self.B, max_tokens + 1, dtype=torch.long, device=self.dev)
        saved = [s0.clone() for s0, _ in self.states]
        with torch.cuda.stream(self.stream):
            self._reset()
            self._two_steps()
            self.stream.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=self.stream):
                self._two_steps()
        torch.cuda.current_stream(self.dev).wait_stream(self.stream)
        for (s0, _), s in zip(self.states, saved):
            s0.copy_(s)
        self._saved = saved

    def _reset(self):
        self.pos.fill_(self.prompt_len)
        self.count.zero_()
        self.tok.copy_(sample_tokens(self.first_logits, self.temperature, self.top_k)[:, None])

    @torch.no_grad()
    def generate(self, n: int) -> torch.Tensor:
        if self.graph is None:
            self.capture(n)
        if n % 2 or n + 1 > self.out.shape[1]:
            raise ValueError("n must be even and at most the captured length")
        cur = torch.cuda.current_stream(self.dev)
        self.stream.wait_stream(cur)
        with torch.cuda.stream(self.stream):
            for (s0, _), s in zip(self.states, self._saved):
                s0.copy_(s)
            self._reset()
            first = self.tok.clone()
            for _ in range(n // 2):
                self.graph.replay()
        cur.wait_stream(self.stream)
        return torch.cat([first, self.out[:, :n]], dim=1)

    def release(self):
        self.graph = None
