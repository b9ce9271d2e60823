"""Llama-style decoder for the FP8 training config (BASELINE cfg5).

8 layers, dim 4096, 32 heads, SwiGLU ffn 14336, vocab 32000, RMSNorm and
RoPE; every attention / MLP projection is an :class:`FP8BlockLinear`
(per-block FP8 forward, dgrad and wgrad).  The token embedding and the LM
head stay bf16: the head's 32000 output rows do not split into whole
128-row tiles across 8 ranks (4000 rows each), which the per-block FP8
all-gather requires.  Attention itself runs in bf16 through
``scaled_dot_product_attention`` (it is not a linear layer).  Weights are
random-init; inputs are synthetic token ids.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .fp8_linear import FP8BlockLinear


@dataclass
class LlamaConfig:
    n_layers: int = 8
    dim: int = 4096
    n_heads: int = 32
    ffn_dim: int = 14336
    vocab: int = 32000
    seq_len: int = 4096
    norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    linear_scaling: str = "fp32"  # FP8BlockLinear.scaling: "fp32" or "e8m0"

    def linear_params(self) -> int:
        """Parameters in linear layers incl. the LM head (the FLOP basis)."""
        per_layer = 4 * self.dim * self.dim + 3 * self.dim * self.ffn_dim
        return self.n_layers * per_layer + self.dim * self.vocab


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).to(x.dtype) * self.weight.to(x.dtype)


def rope_tables(cfg: LlamaConfig, device):
    hd = cfg.dim // cfg.n_heads
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, hd, 2, device=device, dtype=torch.float32) / hd))
    t = torch.arange(cfg.seq_len, device=device, dtype=torch.float32)
    f = torch.outer(t, inv)
    return f.cos(), f.sin()


def apply_rope(x, cos, sin):
    # x [B, H, T, hd]; rotate (even, odd) pairs.
    x1, x2 = x[..., 0::2], x[..., 1::2]
    c, s = cos[: x.shape[-2]], sin[: x.shape[-2]]
    out = torch.stack((x1 * c - x2 * s, x1 * s + x2 * c), dim=-1)
    return out.flatten(-2).to(x.dtype)


class Block(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        d, f = cfg.dim, cfg.ffn_dim
        self.n_heads = cfg.n_heads
        self.attn_norm = RMSNorm(d, cfg.norm_eps)
        self.wq = FP8BlockLinear(d, d, bias=False)
        self.wk = FP8BlockLinear(d, d, bias=False)
        self.wv = FP8BlockLinear(d, d, bias=False)
        self.wo = FP8BlockLinear(d, d, bias=False)
        self.mlp_norm = RMSNorm(d, cfg.norm_eps)
        self.w1 = FP8BlockLinear(d, f, bias=False)
        self.w3 = FP8BlockLinear(d, f, bias=False)
        self.w2 = FP8BlockLinear(f, d, bias=False)
        for lin in (self.wq, self.wk, self.wv, self.wo, self.w1, self.w3, self.w2):
            lin.scaling = cfg.linear_scaling

    def forward(self, x, cos, sin):
        b, t, d = x.shape
        h = self.attn_norm(x)
        hd = d // self.n_heads
        q = self.wq(h).view(b, t, self.n_heads, hd).transpose(1, 2)
        k = self.wk(h).view(b, t, self.n_heads, hd).transpose(1, 2)
        v = self.wv(h).view(b, t, self.n_heads, hd).transpose(1, 2)
        q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + self.wo(a.transpose(1, 2).reshape(b, t, d))
        h = self.mlp_norm(x)
        return x + self.w2(F.silu(self.w1(h)) * self.w3(h))


class Llama(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.cfg = cfg
        self.embed = nn.Embedding(cfg.vocab, cfg.dim)
        self.layers = nn.ModuleList(Block(cfg) for _ in range(cfg.n_layers))
        self.norm = RMSNorm(cfg.dim, cfg.norm_eps)
        self.head = nn.Linear(cfg.dim, cfg.vocab, bias=False)

    def init_weights(self, seed: int = 0):
        g = torch.Generator(device=self.embed.weight.device).manual_seed(seed)
        with torch.no_grad():
            for p in self.parameters():
                if p.ndim == 2:
                    t = getattr(p, "_tensor", p)
                    t.normal_(0.0, 0.02, generator=g)

    def forward(self, tokens):
        x = self.embed(tokens)
        cos, sin = rope_tables(self.cfg, tokens.device)
        for layer in self.layers:
            x = layer(x, cos, sin)
        return self.head(self.norm(x))
