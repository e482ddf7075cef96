"""Llama decoder block workload (the model ``compile_model`` is benchmarked on).

Same module tree, parameter names, creation order and seeded initialisation
as the reference workload (models/llama_block.py:27-159), so
``build_llama_block(cfg, seed)`` reproduces the reference weights bit for bit
when the extensions are off.  Extensions (BASELINE configs C1/C3):

* ``kv_heads``: grouped-query attention (k/v project to kv_heads*head_dim);
  ``None`` = multi-head, the reference behaviour.
* ``causal``: lower-triangular attention mask; ``False`` = the reference's
  unmasked softmax (llama_block.py:101-102).

The forward is written with explicit ATen-level math (no fused SDPA) so that
``torch.export`` yields the core ops the capture stage maps.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import nn


@dataclass
class LlamaBlockConfig:
    batch: int = 2
    seq: int = 256
    hidden: int = 256
    heads: int = 4
    intermediate: int = 512
    eps: float = 1e-5
    rope_theta: float = 10000.0
    dtype: torch.dtype = torch.float16
    kv_heads: int | None = None
    causal: bool = False

    @property
    def head_dim(self) -> int:
        if self.hidden % self.heads:
            raise ValueError("hidden must be a multiple of heads")
        return self.hidden // self.heads

    @property
    def n_kv(self) -> int:
        return self.heads if self.kv_heads is None else self.kv_heads

    @property
    def tokens(self) -> int:
        return self.batch * self.seq


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float, dtype: torch.dtype) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim, dtype=dtype))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def rope_tables(seq: int, head_dim: int, theta: float, dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin tables [seq, head_dim]: angles in fp32, then cast to ``dtype``."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    ang = torch.outer(torch.arange(seq, dtype=torch.float32), inv)
    ang = torch.cat((ang, ang), dim=-1)
    return ang.cos().to(dtype), ang.sin().to(dtype)


class LlamaAttention(nn.Module):
    def __init__(self, cfg: LlamaBlockConfig) -> None:
        super().__init__()
        self.heads, self.kv_heads, self.head_dim, self.causal = cfg.heads, cfg.n_kv, cfg.head_dim, cfg.causal
        kv = cfg.n_kv * cfg.head_dim
        self.q_proj = nn.Linear(cfg.hidden, cfg.hidden, bias=False, dtype=cfg.dtype)
        self.k_proj = nn.Linear(cfg.hidden, kv, bias=False, dtype=cfg.dtype)
        self.v_proj = nn.Linear(cfg.hidden, kv, bias=False, dtype=cfg.dtype)
        self.o_proj = nn.Linear(cfg.hidden, cfg.hidden, bias=False, dtype=cfg.dtype)
        if cfg.causal:
            i = torch.arange(cfg.seq)
            # additive mask: 0 on/below the diagonal, -inf above
            mask = torch.zeros(cfg.seq, cfg.seq, dtype=cfg.dtype).masked_fill(i.unsqueeze(0) > i.unsqueeze(1), float("-inf"))
            self.register_buffer("causal_mask", mask)

    def forward(self, h: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        b, s, _ = h.shape
        q = self.q_proj(h).view(b, s, self.heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(h).view(b, s, self.kv_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(h).view(b, s, self.kv_heads, self.head_dim).transpose(1, 2)
        q = q * cos + rotate_half(q) * sin
        k = k * cos + rotate_half(k) * sin
        if self.kv_heads != self.heads:
            rep = self.heads // self.kv_heads
            k = k[:, :, None].expand(b, self.kv_heads, rep, s, self.head_dim).reshape(b, self.heads, s, self.head_dim)
            v = v[:, :, None].expand(b, self.kv_heads, rep, s, self.head_dim).reshape(b, self.heads, s, self.head_dim)
        scores = torch.matmul(q, k.transpose(-1, -2)) * (self.head_dim ** -0.5)
        if self.causal:
            scores = scores + self.causal_mask
        a = torch.matmul(torch.softmax(scores, dim=-1), v)
        return self.o_proj(a.transpose(1, 2).reshape(b, s, self.heads * self.head_dim))


class LlamaMLP(nn.Module):
    def __init__(self, cfg: LlamaBlockConfig) -> None:
        super().__init__()
        self.gate_proj = nn.Linear(cfg.hidden, cfg.intermediate, bias=False, dtype=cfg.dtype)
        self.up_proj = nn.Linear(cfg.hidden, cfg.intermediate, bias=False, dtype=cfg.dtype)
        self.down_proj = nn.Linear(cfg.intermediate, cfg.hidden, bias=False, dtype=cfg.dtype)

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        return self.down_proj(torch.nn.functional.silu(self.gate_proj(h)) * self.up_proj(h))


class LlamaBlock(nn.Module):
    """``forward(x)``, ``x: [B, S, D]`` -> ``[B, S, D]``."""

    def __init__(self, cfg: LlamaBlockConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.input_norm = RMSNorm(cfg.hidden, cfg.eps, cfg.dtype)
        self.attn = LlamaAttention(cfg)
        self.post_norm = RMSNorm(cfg.hidden, cfg.eps, cfg.dtype)
        self.mlp = LlamaMLP(cfg)
        cos, sin = rope_tables(cfg.seq, cfg.head_dim, cfg.rope_theta, cfg.dtype)
        self.register_buffer("rope_cos", cos)
        self.register_buffer("rope_sin", sin)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x + self.attn(self.input_norm(x), self.rope_cos, self.rope_sin)
        return x + self.mlp(self.post_norm(x))

    def example_inputs(self, seed: int | None = None) -> tuple[torch.Tensor]:
        if seed is not None:
            torch.manual_seed(seed)
        c = self.cfg
        return (torch.randn(c.batch, c.seq, c.hidden, dtype=c.dtype),)


def build_llama_block(cfg: LlamaBlockConfig | None = None, seed: int = 0) -> LlamaBlock:
    """Deterministic weights: 2-D weights ~ N(0, 0.02), norm gains ~ U(0.8, 1.2)
    (the reference's init, llama_block.py:148-159)."""
    cfg = cfg or LlamaBlockConfig()
    torch.manual_seed(seed)
    block = LlamaBlock(cfg)
    with torch.no_grad():
        for _, p in block.named_parameters():
            if p.ndim == 2:
                p.normal_(0.0, 0.02)
            else:
                p.uniform_(0.8, 1.2)
    return block.eval()
