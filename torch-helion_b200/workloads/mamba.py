"""Mamba-2 (SSD) backbone workload.

Same module tree, parameter names, creation order and seeded initialisation
as the reference workload (models/mamba.py:73-391), so
``build_mamba_model(cfg, seed)`` reproduces the reference weights when the
extensions are off.  The mixer evaluates the scan in the reference's
``chunked`` form (mamba.py:163-223) or its ``quadratic`` dual (:226-251).

Extensions (BASELINE configs C2/C4), all off by default:
* ``vocab``: an input token embedding (registered last, so the shared
  parameters keep the reference's random stream) and ``tie_lm_head`` to
  return tied-embedding logits instead of the final-norm hidden state.
* :func:`apply_baseline_init`: the BASELINE A distribution
  A = -exp(U[log 1, log 16]) (the reference draws A in [-1, -0.1]).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import nn


@dataclass
class MambaConfig:
    batch: int = 2
    seq: int = 256
    d_model: int = 512
    expand: int = 2
    headdim: int = 32
    d_state: int = 32
    chunk: int = 64
    n_layers: int = 2
    mode: str = "quadratic"
    ngroups: int | None = None
    d_conv: int = 4
    use_conv: bool = False
    eps: float = 1e-5
    dt_min: float = 0.001
    dt_max: float = 0.1
    dtype: torch.dtype = torch.float16
    vocab: int | None = None
    tie_lm_head: bool = False

    @property
    def d_inner(self) -> int:
        return self.expand * self.d_model

    @property
    def nheads(self) -> int:
        if self.d_inner % self.headdim:
            raise ValueError("d_inner must be a multiple of headdim")
        return self.d_inner // self.headdim

    @property
    def groups(self) -> int:
        return self.nheads if self.ngroups is None else self.ngroups

    @property
    def d_bc(self) -> int:
        return self.groups * self.d_state

    @property
    def d_in_proj(self) -> int:
        return 2 * self.d_inner + 2 * self.d_bc + self.nheads

    @property
    def tokens(self) -> int:
        return self.batch * self.seq

    @property
    def nchunks(self) -> int:
        if self.seq % self.chunk:
            raise ValueError("seq must be a multiple of chunk")
        return self.seq // self.chunk


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float, dtype: torch.dtype) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim, dtype=dtype))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight


def chunk_masks(chunk: int, nchunks: int, dtype: torch.dtype):
    """(within [l,l] j<=i, across [c,c] c<z, prefix [l,l] j<=i as a right-multiplied running sum)."""
    i = torch.arange(chunk)
    within = (i.unsqueeze(1) >= i.unsqueeze(0)).to(dtype)
    prefix = (i.unsqueeze(1) <= i.unsqueeze(0)).to(dtype)
    c = torch.arange(nchunks)
    across = (c.unsqueeze(1) > c.unsqueeze(0)).to(dtype)
    return within, across, prefix


def scan_chunked(x, dA, dt, B, C, within, across, prefix):
    """Chunk-major operands [b,h,c,l,...]; four steps: running decay, diagonal
    block, chunk states, inter-chunk recurrence (mamba.py:163-223)."""
    n = B.shape[-1]
    cum = torch.matmul(dA.unsqueeze(-2), prefix).squeeze(-2)
    last = cum[..., -1:]
    gram = torch.matmul(C, B.transpose(-1, -2))
    decay = torch.exp((cum.unsqueeze(-1) - cum.unsqueeze(-2)) * within) * within
    y_diag = torch.matmul(gram * decay * dt.unsqueeze(-2), x)
    weights = (dt * torch.exp(last - cum)).unsqueeze(-1)
    states = torch.matmul((x * weights).transpose(-1, -2), B)
    tot = last.squeeze(-1)
    run = torch.matmul(tot.unsqueeze(-2), prefix[: tot.shape[-1], : tot.shape[-1]]).squeeze(-2)
    dec_c = torch.exp(((run - tot).unsqueeze(-1) - run.unsqueeze(-2)) * across) * across
    carried = torch.matmul(dec_c, states.flatten(-2)).unflatten(-1, (x.shape[-1], n))
    y_off = torch.matmul(C, carried.transpose(-1, -2)) * torch.exp(cum).unsqueeze(-1)
    return y_diag + y_off


def scan_quadratic(x, dA, dt, B, C, causal):
    """Head-major operands [b,h,s,...]; decay-masked attention dual (mamba.py:226-251)."""
    cum = torch.cumsum(dA, dim=-1)
    gram = torch.matmul(C, B.transpose(-1, -2))
    delta = (cum.unsqueeze(-1) - cum.unsqueeze(-2)) * causal
    return torch.matmul(gram * torch.exp(delta) * causal * dt.unsqueeze(-2), x)


class Mamba2Mixer(nn.Module):
    def __init__(self, cfg: MambaConfig) -> None:
        super().__init__()
        self.cfg = cfg
        d = cfg.dtype
        self.in_proj = nn.Linear(cfg.d_model, cfg.d_in_proj, bias=False, dtype=d)
        self.out_proj = nn.Linear(cfg.d_inner, cfg.d_model, bias=False, dtype=d)
        self.norm = RMSNorm(cfg.d_inner, cfg.eps, d)
        self.A_log = nn.Parameter(torch.zeros(cfg.nheads, dtype=d))
        self.D = nn.Parameter(torch.ones(cfg.nheads, dtype=d))
        self.dt_bias = nn.Parameter(torch.zeros(cfg.nheads, dtype=d))
        if cfg.use_conv:
            self.conv_weight = nn.Parameter(torch.zeros(cfg.d_inner + 2 * cfg.d_bc, cfg.d_conv, dtype=d))
        within, across, prefix = chunk_masks(cfg.chunk, cfg.nchunks, d)
        self.register_buffer("mask_within", within)
        self.register_buffer("mask_across", across)
        self.register_buffer("mask_prefix", prefix)
        i = torch.arange(cfg.seq)
        self.register_buffer("mask_causal", (i.unsqueeze(1) >= i.unsqueeze(0)).to(d))
        self.register_buffer("mask_seq_prefix", (i.unsqueeze(1) <= i.unsqueeze(0)).to(d))

    def _conv(self, xbc: torch.Tensor) -> torch.Tensor:
        width = xbc.shape[-1]
        padded = torch.nn.functional.pad(xbc.transpose(1, 2), (self.cfg.d_conv - 1, 0))
        out = torch.nn.functional.conv1d(padded, self.conv_weight.unsqueeze(1), groups=width)
        return torch.nn.functional.silu(out.transpose(1, 2))

    def forward(self, u: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        b, s, _ = u.shape
        h, p, n, g = cfg.nheads, cfg.headdim, cfg.d_state, cfg.groups
        z, xbc, dt = torch.split(self.in_proj(u), [cfg.d_inner, cfg.d_inner + 2 * cfg.d_bc, h], dim=-1)
        if cfg.use_conv:
            xbc = self._conv(xbc)
        x, B, C = torch.split(xbc, [cfg.d_inner, cfg.d_bc, cfg.d_bc], dim=-1)
        dt = torch.nn.functional.softplus(dt + self.dt_bias)
        A = -torch.exp(self.A_log)
        if cfg.mode == "chunked":
            c, l = cfg.nchunks, cfg.chunk
            xc = x.reshape(b, c, l, h, p).permute(0, 3, 1, 2, 4)
            Bc = B.reshape(b, c, l, g, n).permute(0, 3, 1, 2, 4)
            Cc = C.reshape(b, c, l, g, n).permute(0, 3, 1, 2, 4)
            dtc = dt.reshape(b, c, l, h).permute(0, 3, 1, 2)
            if g != h:
                Bc, Cc = Bc.expand(b, h, c, l, n), Cc.expand(b, h, c, l, n)
            y = scan_chunked(xc, dtc * A.reshape(1, h, 1, 1), dtc, Bc, Cc, self.mask_within, self.mask_across, self.mask_prefix)
            y = (y + xc * self.D.reshape(1, h, 1, 1, 1)).permute(0, 2, 3, 1, 4).reshape(b, s, cfg.d_inner)
        else:
            xq = x.reshape(b, s, h, p).permute(0, 2, 1, 3)
            Bq = B.reshape(b, s, g, n).permute(0, 2, 1, 3)
            Cq = C.reshape(b, s, g, n).permute(0, 2, 1, 3)
            dtq = dt.permute(0, 2, 1)
            if g != h:
                Bq, Cq = Bq.expand(b, h, s, n), Cq.expand(b, h, s, n)
            y = scan_quadratic(xq, dtq * A.reshape(1, h, 1), dtq, Bq, Cq, self.mask_causal)
            y = (y + xq * self.D.reshape(1, h, 1, 1)).permute(0, 2, 1, 3).reshape(b, s, cfg.d_inner)
        return self.out_proj(self.norm(y * torch.nn.functional.silu(z)))


class Mamba2Block(nn.Module):
    def __init__(self, cfg: MambaConfig) -> None:
        super().__init__()
        self.norm = RMSNorm(cfg.d_model, cfg.eps, cfg.dtype)
        self.mixer = Mamba2Mixer(cfg)

    def forward(self, u: torch.Tensor) -> torch.Tensor:
        return u + self.mixer(self.norm(u))


class MambaModel(nn.Module):
    """``forward(u)``: ``u [B, S, D]`` floats, or ``[B, S]`` token ids when
    ``cfg.vocab`` is set.  Returns the final-norm hidden state, or logits
    with ``cfg.tie_lm_head``."""

    def __init__(self, cfg: MambaConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.layers = nn.ModuleList([Mamba2Block(cfg) for _ in range(cfg.n_layers)])
        self.norm_f = RMSNorm(cfg.d_model, cfg.eps, cfg.dtype)
        if cfg.vocab is not None:
            self.embedding = nn.Embedding(cfg.vocab, cfg.d_model, dtype=cfg.dtype)

    def forward(self, u: torch.Tensor) -> torch.Tensor:
        if self.cfg.vocab is not None:
            u = self.embedding(u)
        for layer in self.layers:
            u = layer(u)
        u = self.norm_f(u)
        if self.cfg.vocab is not None and self.cfg.tie_lm_head:
            return torch.matmul(u, self.embedding.weight.t())
        return u

    def example_inputs(self, seed: int | None = None) -> tuple[torch.Tensor]:
        if seed is not None:
            torch.manual_seed(seed)
        c = self.cfg
        if c.vocab is not None:
            return (torch.randint(0, c.vocab, (c.batch, c.seq)),)
        return (torch.randn(c.batch, c.seq, c.d_model, dtype=c.dtype),)


def build_mamba_model(cfg: MambaConfig | None = None, seed: int = 0) -> MambaModel:
    """The reference's seeded init (mamba.py:362-384): 2-D weights (not conv)
    ~ N(0, 0.02); A in [-1, -0.1]; dt bias so softplus(dt) is log-uniform in
    [dt_min, dt_max]; D = 1; other vectors ~ U(0.9, 1.1); conv ~ N(0, 0.02)."""
    cfg = cfg or MambaConfig()
    torch.manual_seed(seed)
    model = MambaModel(cfg)
    with torch.no_grad():
        for name, prm in model.named_parameters():
            if prm.ndim == 2 and "conv" not in name:
                prm.normal_(0.0, 0.02)
            elif "A_log" in name:
                prm.copy_(torch.log(torch.rand(prm.shape, dtype=torch.float32) * 0.9 + 0.1).to(prm.dtype))
            elif "dt_bias" in name:
                lo, hi = math.log(cfg.dt_min), math.log(cfg.dt_max)
                dt = (torch.rand(prm.shape, dtype=torch.float32) * (hi - lo) + lo).exp().clamp(min=1e-4)
                prm.copy_((dt + torch.log(-torch.expm1(-dt))).to(prm.dtype))
            elif "D" in name and prm.ndim == 1:
                prm.fill_(1.0)
            elif prm.ndim == 1:
                prm.uniform_(0.9, 1.1)
            else:
                prm.normal_(0.0, 0.02)
    return model.eval()


def build_mamba_block(cfg: MambaConfig | None = None, seed: int = 0) -> MambaModel:
    cfg = cfg or MambaConfig(n_layers=1)
    cfg.n_layers = 1
    return build_mamba_model(cfg, seed)


def apply_baseline_init(model: MambaModel, seed: int = 0) -> MambaModel:
    """A = -exp(U[log 1, log 16]) per head and layer, drawn
    from a private generator so the other weights are untouched."""
    gen = torch.Generator().manual_seed(10_000 + seed)
    with torch.no_grad():
        for name, prm in model.named_parameters():
            if name.endswith("A_log"):
                prm.copy_((torch.rand(prm.shape, generator=gen) * math.log(16.0)).to(prm.dtype))
    return model
