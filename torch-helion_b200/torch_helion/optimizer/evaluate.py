"""Compile-time evaluation of OpGraph nodes with PyTorch.

Used for constant folding of parameter-only sub-graphs and for the
numerical check that every canonicalisation pass preserves the model's
outputs -- the same two roles the reference evaluator has
(src/torch_helion/optimizer/evaluate.py:36-166).  Math runs in fp32.  This
never executes a compiled Program: that is the B200 runtime's job.

Semantics of the B200 macro ops (documented in torch_helion.capture.ops):
``rope``, ``attention`` (+causal, grouped KV), ``ssd`` (+D skip, silu(z)
gate), ``causal_conv1d``, ``rmsnorm``, ``embedding``.
"""

from __future__ import annotations

import math
from typing import Any, Callable

import torch
import torch.nn.functional as F

from ..capture.opgraph import OpGraph


def rope_2d(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, head_dim: int, seq: int) -> torch.Tensor:
    """RoPE on token-major ``[T, H*d]``: x*cos + rotate_half(x)*sin per head,
    position = row % seq, tables ``[seq, d]``."""
    t = x.shape[0]
    xh = x.reshape(t, -1, head_dim)
    half = head_dim // 2
    rot = torch.cat((-xh[..., half:], xh[..., :half]), -1)
    pos = torch.arange(t) % seq
    c = cos.reshape(seq, head_dim)[pos].unsqueeze(1)
    s = sin.reshape(seq, head_dim)[pos].unsqueeze(1)
    return (xh * c + rot * s).reshape(x.shape)


def attention_2d(q, k, v, batch, seq, heads, kv_heads, head_dim, scale, causal):
    q4 = q.reshape(batch, seq, heads, head_dim).transpose(1, 2)
    k4 = k.reshape(batch, seq, kv_heads, head_dim).transpose(1, 2)
    v4 = v.reshape(batch, seq, kv_heads, head_dim).transpose(1, 2)
    if kv_heads != heads:
        k4 = k4.repeat_interleave(heads // kv_heads, 1)
        v4 = v4.repeat_interleave(heads // kv_heads, 1)
    s = (q4 @ k4.transpose(-1, -2)) * scale
    if causal:
        s = s.masked_fill(torch.triu(torch.ones(seq, seq, dtype=torch.bool), 1), float("-inf"))
    return (torch.softmax(s, -1) @ v4).transpose(1, 2).reshape(batch * seq, heads * head_dim)


def ssd_2d(x, dt, A, B, C, D, z, batch, seq, heads, head_dim, ngroups, state_dim, chunk=256):
    """Token-major Mamba-2 scan (see torch_helion.capture.ops ``ssd``):
    y = SSD(x, dt*A, dt, B, C) + D*x, then y*silu(z) when z is given."""
    b, s, h, p, g, n = batch, seq, heads, head_dim, ngroups, state_dim
    xh = x.reshape(b, s, h, p).permute(0, 2, 1, 3)
    Bh = B.reshape(b, s, g, n).permute(0, 2, 1, 3).repeat_interleave(h // g, 1)
    Ch = C.reshape(b, s, g, n).permute(0, 2, 1, 3).repeat_interleave(h // g, 1)
    dth = dt.reshape(b, s, h).permute(0, 2, 1)
    dA = dth * A.reshape(1, h, 1)
    L = min(chunk, s)
    pad = (-s) % L
    if pad:
        xh, Bh, Ch = (F.pad(t, (0, 0, 0, pad)) for t in (xh, Bh, Ch))
        dA, dth = F.pad(dA, (0, pad)), F.pad(dth, (0, pad))
    c = (s + pad) // L
    xc, Bc, Cc = xh.reshape(b, h, c, L, p), Bh.reshape(b, h, c, L, n), Ch.reshape(b, h, c, L, n)
    dAc, dtc = dA.reshape(b, h, c, L), dth.reshape(b, h, c, L)
    cum = torch.cumsum(dAc, -1)
    i = torch.arange(L)
    low = i.unsqueeze(1) >= i.unsqueeze(0)
    decay = torch.exp((cum.unsqueeze(-1) - cum.unsqueeze(-2)).masked_fill(~low, 0.0)) * low
    y = ((Cc @ Bc.transpose(-1, -2)) * decay * dtc.unsqueeze(-2)) @ xc
    states = (xc * (dtc * torch.exp(cum[..., -1:] - cum)).unsqueeze(-1)).transpose(-1, -2) @ Bc
    run = torch.zeros(b, h, p, n, dtype=x.dtype)
    carried = torch.empty_like(states)
    for zc in range(c):
        carried[:, :, zc] = run
        run = torch.exp(cum[:, :, zc, -1]).reshape(b, h, 1, 1) * run + states[:, :, zc]
    y = y + (Cc @ carried.transpose(-1, -2)) * torch.exp(cum).unsqueeze(-1)
    y = y.reshape(b, h, c * L, p)[:, :, :s].permute(0, 2, 1, 3).reshape(b * s, h * p)
    if D is not None:
        y = y + x * D.reshape(-1).repeat_interleave(p).reshape(1, -1)
    if z is not None:
        y = y * F.silu(z)
    return y


def causal_conv1d_2d(x, w, batch, seq, act):
    ch = x.shape[-1]
    k = w.shape[-1]
    xt = x.reshape(batch, seq, ch).transpose(1, 2)
    y = F.conv1d(F.pad(xt, (k - 1, 0)), w.reshape(ch, 1, k), groups=ch).transpose(1, 2).reshape(batch * seq, ch)
    return F.silu(y) if act == "silu" else y


# ----------------------------------------------------------- op semantics
# One function per OpGraph op (or family of ops), registered under the op
# names it defines.  Each takes the operands (floating ones promoted to
# fp32) and the node's attributes.
_SEMANTICS: dict[str, Callable[[list[torch.Tensor], dict[str, Any]], torch.Tensor]] = {}


def _defines(*ops: str):
    def register(fn):
        for op in ops:
            _SEMANTICS[op] = fn
        return fn

    return register


_BINARY_FN = {"add": torch.add, "sub": torch.sub, "mul": torch.mul, "div": torch.div, "max": torch.maximum,
              "powf": torch.pow}


def _binary(op: str):
    fn = _BINARY_FN[op]

    def run(xs, attrs):
        if "scalar" not in attrs:
            return fn(xs[0], xs[1])
        scalar = torch.tensor(float(attrs["scalar"]), dtype=xs[0].dtype)
        # a scalar operand that came first in the source expression keeps its place (sub, div, pow)
        return fn(scalar, xs[0]) if attrs.get("scalar_first") else fn(xs[0], scalar)

    return run


for _op in _BINARY_FN:
    _SEMANTICS[_op] = _binary(_op)

_UNARY_FN = {"exp": torch.exp, "log": torch.log, "neg": torch.neg, "rsqrt": torch.rsqrt, "sqrt": torch.sqrt,
             "sigmoid": torch.sigmoid, "silu": F.silu, "tanh": torch.tanh, "log1p": torch.log1p,
             "softplus": F.softplus, "erf": torch.erf, "square": torch.square}
for _op, _fn in _UNARY_FN.items():
    _SEMANTICS[_op] = (lambda f: (lambda xs, attrs: f(xs[0])))(_fn)


@_defines("gelu")
def _gelu(xs, attrs):
    return F.gelu(xs[0], approximate=attrs.get("approximate", "none"))


def _reduction(name: str):
    how = {"row_sum": torch.sum, "row_max": torch.amax, "row_mean": torch.mean}[name]
    return lambda xs, attrs: how(xs[0], dim=-1, keepdim=attrs.get("keepdim", True))


for _op in ("row_sum", "row_max", "row_mean"):
    _SEMANTICS[_op] = _reduction(_op)


@_defines("row_sumsq")
def _row_sumsq(xs, attrs):
    return xs[0].square().sum(dim=-1, keepdim=True)


@_defines("row_cumsum")
def _row_cumsum(xs, attrs):
    return xs[0].cumsum(dim=-1)


@_defines("cmp_gt")
def _cmp_gt(xs, attrs):
    rhs = float(attrs["scalar"]) if "scalar" in attrs else xs[1]
    return torch.gt(xs[0], rhs)


@_defines("select")
def _select(xs, attrs):
    return torch.where(xs[0].bool(), xs[1], xs[2])


@_defines("softmax")
def _softmax(xs, attrs):
    return xs[0].softmax(dim=-1)


@_defines("matmul")
def _matmul(xs, attrs):
    return torch.matmul(xs[0], xs[1])


@_defines("batch_matmul")
def _bmm(xs, attrs):
    return torch.bmm(xs[0], xs[1])


@_defines("broadcast", "expand")
def _expand(xs, attrs):
    return xs[0].expand(*attrs["shape"])


@_defines("view")
def _view(xs, attrs):
    return xs[0].reshape(*attrs["shape"])


@_defines("permute")
def _permute(xs, attrs):
    return xs[0].permute(*attrs["dims"])


@_defines("clone", "cast")
def _copy(xs, attrs):
    return xs[0].clone()


@_defines("slice")
def _slice(xs, attrs):
    lo, hi = attrs["start"], attrs["end"]
    return xs[0].narrow(attrs["dim"], lo, hi - lo)


@_defines("cat")
def _cat(xs, attrs):
    return torch.cat(list(xs), dim=attrs["dim"])


@_defines("pad")
def _pad(xs, attrs):
    return F.pad(xs[0], list(attrs["pad"]), value=attrs.get("value", 0.0))


@_defines("conv1d")
def _conv1d(xs, attrs):
    bias = xs[2] if len(xs) > 2 else None
    return F.conv1d(xs[0], xs[1], bias, stride=attrs["stride"], padding=attrs["padding"],
                    dilation=attrs["dilation"], groups=attrs["groups"])


@_defines("embedding")
def _embedding(xs, attrs):
    ids, table = xs
    return table.index_select(0, ids.long().reshape(-1)).reshape(*ids.shape, table.shape[-1])


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    lo, hi = x.chunk(2, dim=-1)
    return torch.cat((hi.neg(), lo), dim=-1)


@_defines("rotate_half")
def _rotate(xs, attrs):
    return _rotate_half(xs[0])


@_defines("rmsnorm")
def _rmsnorm(xs, attrs):
    x, gain = xs
    return x * (x.square().mean(dim=-1, keepdim=True) + attrs["eps"]).rsqrt() * gain.reshape(-1)


@_defines("rope")
def _rope(xs, attrs):
    if "seq" in attrs:
        return rope_2d(xs[0], xs[1], xs[2], attrs["head_dim"], attrs["seq"])
    x, cos, sin = xs  # head-split form: tables broadcast over batch and heads
    return x * cos + _rotate_half(x) * sin


@_defines("attention")
def _attention(xs, a):
    return attention_2d(xs[0], xs[1], xs[2], a["batch"], a["seq"], a["heads"], a.get("kv_heads", a["heads"]),
                        a["head_dim"], a["scale"], a.get("causal", False))


@_defines("ssd")
def _ssd(xs, a):
    x, dt, A, B, C, *extra = xs
    D = extra.pop(0) if a.get("has_D") else None
    z = extra.pop(0) if a.get("gate") else None
    return ssd_2d(x, dt, A, B, C, D, z, a["batch"], a["seq"], a["heads"], a["head_dim"], a["ngroups"],
                  a["state_dim"], a.get("chunk", 256))


@_defines("causal_conv1d")
def _causal_conv(xs, attrs):
    return causal_conv1d_2d(xs[0], xs[1], attrs["batch"], attrs["seq"], attrs.get("act"))


def eval_op(op: str, args: list[torch.Tensor], attrs: dict[str, Any]) -> torch.Tensor:
    """The fp32 value of ``op(args)`` (integer and boolean operands pass
    through unchanged)."""
    fn = _SEMANTICS.get(op)
    if fn is None:
        raise NotImplementedError(f"eval_op: {op}")
    return fn([t.float() if t.is_floating_point() else t for t in args], attrs)


def evaluate_graph(graph: OpGraph, inputs, keep_float32: bool = True, upto: set[str] | None = None) -> dict[str, torch.Tensor]:
    if isinstance(inputs, (list, tuple)):
        inputs = dict(zip(graph.inputs, inputs))
    env: dict[str, torch.Tensor] = {}
    for node in graph:
        if node.kind == "input":
            env[node.name] = inputs[node.name].reshape(node.type.shape)
        elif node.kind in ("param", "const"):
            env[node.name] = graph.value(node.name)
        else:
            out = eval_op(node.op, [env[i] for i in node.inputs], node.attrs)
            if tuple(out.shape) != node.type.shape:
                out = out.reshape(node.type.shape)
            env[node.name] = out if keep_float32 else out.to(node.type.torch_dtype)
    return env


def graph_outputs(graph: OpGraph, inputs) -> list[torch.Tensor]:
    env = evaluate_graph(graph, inputs)
    return [env[o] for o in graph.outputs]


def max_rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    """The reference metric: max|a-b| / max|b| (evaluate.py:174-176)."""
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / (b.abs().max() + 1e-6))


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double().reshape(-1), b.double().reshape(-1)
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


__all__ = ["eval_op", "evaluate_graph", "graph_outputs", "max_rel_err", "rel_l2", "rope_2d", "attention_2d", "ssd_2d",
           "causal_conv1d_2d", "math"]
