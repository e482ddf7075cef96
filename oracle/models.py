"""Eager forwards of the reference workloads, restated functionally -- test
infrastructure (see ``oracle/__init__.py``).

Every function takes a parameter dict whose keys are the reference modules'
``state_dict`` names, so a state dict saved from the reference model (golden
fixtures) or from any structurally identical module can be fed in as is.
All math runs in ``dtype`` (fp32 by default) on the CPU; pass bf16-rounded
weights/inputs to get the "fp32 eager on bf16-rounded operands" oracle.

Extensions beyond the reference (each defaults to the reference behaviour):
* Llama: ``kv_heads`` (grouped-query attention) and ``causal`` masking;
  the reference block is MHA and non-causal (models/llama_block.py:87-102).
* Mamba: an input ``embedding`` (token ids -> d_model) and an optional
  tied LM head; the reference backbone takes float embeddings
  (models/mamba.py:343-359).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .ssd import ssd_chunked, ssd_quadratic


def _p(params, name, dtype):
    return params[name].to(dtype)


def rmsnorm(x, weight, eps):
    """models/llama_block.py:61-63 and models/mamba.py:138-140."""
    var = x.pow(2).mean(-1, keepdim=True)
    return x * torch.rsqrt(var + eps) * weight


def rotate_half(x):
    """models/llama_block.py:66-70."""
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def rope_tables(seq, head_dim, theta, dtype):
    """models/llama_block.py:73-79: fp32 angles, then cast to the model dtype."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    freqs = torch.outer(torch.arange(seq, dtype=torch.float32), inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def llama_block_forward(params, x, *, heads, kv_heads=None, eps, rope_theta=10000.0, causal=False,
                        model_dtype=torch.float32, dtype=torch.float32, prefix=""):
    """LlamaBlock.forward (models/llama_block.py:138-141): pre-norm attention
    with RoPE (:92-105) and a SwiGLU MLP (:115-116), both residual.

    ``model_dtype`` is the dtype the reference builds its RoPE tables in
    (they are rounded to it, llama_block.py:79); ``dtype`` is the math dtype.
    """
    kv_heads = kv_heads or heads
    P = lambda n: _p(params, prefix + n, dtype)
    x = x.to(dtype)
    b, s, d_model = x.shape
    hd = d_model // heads
    cos, sin = rope_tables(s, hd, rope_theta, model_dtype)
    cos, sin = cos.to(dtype), sin.to(dtype)
    h = rmsnorm(x, P("input_norm.weight"), eps)
    q = (h @ P("attn.q_proj.weight").t()).view(b, s, heads, hd).transpose(1, 2)
    k = (h @ P("attn.k_proj.weight").t()).view(b, s, kv_heads, hd).transpose(1, 2)
    v = (h @ P("attn.v_proj.weight").t()).view(b, s, kv_heads, hd).transpose(1, 2)
    q = q * cos + rotate_half(q) * sin
    k = k * cos + rotate_half(k) * sin
    if kv_heads != heads:
        k = k.repeat_interleave(heads // kv_heads, 1)
        v = v.repeat_interleave(heads // kv_heads, 1)
    scores = (q @ k.transpose(-1, -2)) * (hd ** -0.5)
    if causal:
        scores = scores.masked_fill(torch.triu(torch.ones(s, s, dtype=torch.bool), 1), float("-inf"))
    a = (torch.softmax(scores, -1) @ v).transpose(1, 2).reshape(b, s, heads * hd)
    x = x + a @ P("attn.o_proj.weight").t()
    h2 = rmsnorm(x, P("post_norm.weight"), eps)
    mlp = (F.silu(h2 @ P("mlp.gate_proj.weight").t()) * (h2 @ P("mlp.up_proj.weight").t())) @ P("mlp.down_proj.weight").t()
    return x + mlp


def mamba_mixer_forward(params, u, *, d_inner, nheads, headdim, d_state, ngroups, chunk, eps, use_conv, d_conv,
                        mode="chunked", dtype=torch.float32, prefix=""):
    """Mamba2Mixer.forward (models/mamba.py:285-328)."""
    P = lambda n: _p(params, prefix + n, dtype)
    b, s, _ = u.shape
    h, p, n, g = nheads, headdim, d_state, ngroups
    d_bc = g * n
    proj = u @ P("in_proj.weight").t()
    z, xbc, dt = torch.split(proj, [d_inner, d_inner + 2 * d_bc, h], dim=-1)
    if use_conv:                                                   # mamba.py:278-283
        w = P("conv_weight")
        pad = F.pad(xbc.transpose(1, 2), (d_conv - 1, 0))
        xbc = F.silu(F.conv1d(pad, w.unsqueeze(1), groups=xbc.shape[-1]).transpose(1, 2))
    x, B, C = torch.split(xbc, [d_inner, d_bc, d_bc], dim=-1)
    dt = F.softplus(dt + P("dt_bias"))                             # mamba.py:297
    A = -torch.exp(P("A_log"))                                     # mamba.py:298
    xh = x.reshape(b, s, h, p).permute(0, 2, 1, 3)
    Bh = B.reshape(b, s, g, n).permute(0, 2, 1, 3).repeat_interleave(h // g, 1)
    Ch = C.reshape(b, s, g, n).permute(0, 2, 1, 3).repeat_interleave(h // g, 1)
    dth = dt.permute(0, 2, 1)
    dA = dth * A.reshape(1, h, 1)
    if mode == "chunked":
        y = ssd_chunked(xh, dA, dth, Bh, Ch, chunk)
    else:
        y = ssd_quadratic(xh, dA, dth, Bh, Ch)
    y = y + xh * P("D").reshape(1, h, 1, 1)
    y = y.permute(0, 2, 1, 3).reshape(b, s, d_inner)
    gated = rmsnorm(y * F.silu(z), P("norm.weight"), eps)          # mamba.py:327
    return gated @ P("out_proj.weight").t()


def mamba_forward(params, u, *, n_layers, d_model, expand=2, headdim, d_state, ngroups=None, chunk, eps=1e-5,
                  use_conv=False, d_conv=4, mode="chunked", embedding=False, lm_head=False, dtype=torch.float32):
    """MambaModel.forward (models/mamba.py:352-355): residual pre-norm blocks
    (:339-340) and a final norm.  With ``embedding`` the input is token ids
    looked up in ``embedding.weight``; with ``lm_head`` the output is the
    tied-embedding logits."""
    d_inner = expand * d_model
    nheads = d_inner // headdim
    g = nheads if ngroups is None else ngroups
    if embedding:
        x = params["embedding.weight"].to(dtype)[u]
    else:
        x = u.to(dtype)
    for i in range(n_layers):
        pre = f"layers.{i}."
        hn = rmsnorm(x, _p(params, pre + "norm.weight", dtype), eps)
        x = x + mamba_mixer_forward(params, hn, d_inner=d_inner, nheads=nheads, headdim=headdim, d_state=d_state,
                                    ngroups=g, chunk=chunk, eps=eps, use_conv=use_conv, d_conv=d_conv, mode=mode,
                                    dtype=dtype, prefix=pre + "mixer.")
    x = rmsnorm(x, _p(params, "norm_f.weight", dtype), eps)
    if lm_head:
        return x @ params["embedding.weight"].to(dtype).t()
    return x


def round_params(params, dtype):
    """Round every floating tensor to ``dtype`` (the bf16 oracle's operands)."""
    return {k: (v.to(dtype) if v.is_floating_point() else v) for k, v in params.items()}


def max_rel_err(a, b):
    """The reference error metric (src/torch_helion/optimizer/evaluate.py:174-176)."""
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / (b.abs().max() + 1e-6))


def rel_l2(a, b):
    a, b = a.double().reshape(-1), b.double().reshape(-1)
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


__all__ = ["rmsnorm", "rotate_half", "rope_tables", "llama_block_forward", "mamba_mixer_forward", "mamba_forward",
           "round_params", "max_rel_err", "rel_l2", "math"]
