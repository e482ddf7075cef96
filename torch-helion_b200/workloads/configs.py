"""The BASELINE configurations C1-C5 as builders of (model, inputs).

Seeds: weights ``build_*(seed=0)`` (+ the BASELINE A override for Mamba),
inputs ``torch.manual_seed(1)``: N(0, 1) activations, uniform token ids.
All data is synthetic; no dataset is involved.
"""

from __future__ import annotations

import math

import torch

from .llama_block import LlamaBlockConfig, build_llama_block
from .mamba import MambaConfig, apply_baseline_init, build_mamba_model

INPUT_SEED = 1


def c1_llama_fp32() -> LlamaBlockConfig:
    """C1: B1 S128 D512 H8 KV8 d64 F1408 theta 1e4 eps 1e-6 fp32, causal."""
    return LlamaBlockConfig(batch=1, seq=128, hidden=512, heads=8, intermediate=1408, eps=1e-6, rope_theta=10000.0,
                            dtype=torch.float32, kv_heads=8, causal=True)


def c2_mamba_block_bf16() -> MambaConfig:
    """C2: one Mamba-2 block, B4 S2048 d768 expand 2 headdim 64 (24 heads)
    d_state 128 ngroups 1 conv 4 chunk 256, bf16."""
    return MambaConfig(batch=4, seq=2048, d_model=768, expand=2, headdim=64, d_state=128, chunk=256, n_layers=1,
                       mode="chunked", ngroups=1, d_conv=4, use_conv=True, dtype=torch.bfloat16)


def c3_llama8b_bf16(batch: int = 8, seq: int = 4096) -> LlamaBlockConfig:
    """C3: Llama-3-8B geometry block: D4096 Hq32 Hkv8 d128 F14336 theta 5e5, B8 S4096 causal, bf16."""
    return LlamaBlockConfig(batch=batch, seq=seq, hidden=4096, heads=32, intermediate=14336, eps=1e-5,
                            rope_theta=500000.0, dtype=torch.bfloat16, kv_heads=8, causal=True)


def c4_mamba24_bf16(batch: int = 16, seq: int = 2048) -> MambaConfig:
    """C4: 24-layer Mamba-2 backbone, d_model 1024, expand 2, headdim 64,
    d_state 128, chunk 256, vocab 50280 tied embedding, final RMSNorm, B16 S2048."""
    return MambaConfig(batch=batch, seq=seq, d_model=1024, expand=2, headdim=64, d_state=128, chunk=256,
                       n_layers=24, mode="chunked", ngroups=1, d_conv=4, use_conv=True, dtype=torch.bfloat16,
                       vocab=50280, tie_lm_head=False)


C5_GRID = {"nheads": 64, "headdim": 64, "d_state": (64, 128, 256), "seq": (512, 2048, 8192, 16384), "batch": 8,
           "chunk": 256, "ngroups": 1}


def build(cfg, seed: int = 0):
    if isinstance(cfg, LlamaBlockConfig):
        return build_llama_block(cfg, seed)
    model = build_mamba_model(cfg, seed)
    return apply_baseline_init(model, seed)


def inputs(model, seed: int = INPUT_SEED):
    return model.example_inputs(seed)


def ssd_inputs(batch: int, seq: int, nheads: int, headdim: int, d_state: int, ngroups: int = 1, seed: int = INPUT_SEED,
               dtype=torch.bfloat16, device="cpu"):
    """C5 synthetic scan operands: x, B, C ~ N(0,1); dt log-uniform in
    [1e-3, 0.1] (softplus already applied); A = -exp(U[0, log 16]); D = 1."""
    g = torch.Generator().manual_seed(seed)
    t = batch * seq
    x = torch.randn(t, nheads * headdim, generator=g).to(dtype)
    B = torch.randn(t, ngroups * d_state, generator=g).to(dtype)
    C = torch.randn(t, ngroups * d_state, generator=g).to(dtype)
    dt = torch.exp(torch.rand(t, nheads, generator=g) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3))
    A = -torch.exp(torch.rand(nheads, generator=g) * math.log(16.0))
    D = torch.ones(nheads)
    return {k: v.to(device) for k, v in dict(x=x, B=B, C=C, dt=dt, A=A, D=D).items()}
