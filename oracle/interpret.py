"""CPU interpreter of a B200 OpIR Program -- TEST INFRASTRUCTURE ONLY.

Restates, kernel by kernel, what the reference's OpIR interpreter does
(src/torch_helion/codegen/interpret.py:18-77: bind inputs and constants,
run every kernel in order, GEMM kernels as ``acc_i = lhs @ rhs_i`` plus the
``sumsq`` column and the epilogue SSA) for the kernel kinds of the B200
Program.  The math is written here independently of the product (fp64 by
default), so the partitioner's output can be checked against the eager
oracle on the CPU, and sharded programs can be checked against unsharded
ones with gloo ranks.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .ssd import ssd_chunked


def _bin(op, a, b):
    return {"add": torch.add, "sub": torch.sub, "mul": torch.mul, "div": torch.div, "max": torch.maximum,
            "powf": torch.pow}[op](a, b)


def _scalar(op, a, s, first):
    x, y = (s, a) if first else (a, s)
    if op == "add":
        return x + y
    if op == "sub":
        return x - y
    if op == "mul":
        return x * y
    if op == "div":
        return x / y
    if op == "max":
        return torch.clamp_min(a, s)
    if op == "powf":
        return torch.pow(a, s) if not first else torch.pow(torch.full_like(a, s), a)
    raise ValueError(op)


def _rope(x, cos, sin, head_dim, seq):
    t = x.shape[0]
    xh = x.reshape(t, -1, head_dim)
    half = head_dim // 2
    rot = torch.cat((-xh[..., half:], xh[..., :half]), -1)
    pos = torch.arange(t) % seq
    return (xh * cos.reshape(seq, head_dim)[pos, None] + rot * sin.reshape(seq, head_dim)[pos, None]).reshape(x.shape)


def _epilogue_op(op, args, attrs):
    if op in ("add", "sub", "mul", "div", "max", "powf"):
        if "scalar" in attrs:
            return _scalar(op, args[0], float(attrs["scalar"]), bool(attrs.get("scalar_first", False)))
        return _bin(op, args[0], args[1])
    if op == "broadcast":
        return args[0].expand(attrs["shape"])
    if op == "silu":
        return F.silu(args[0])
    if op == "softplus":
        return F.softplus(args[0])
    if op == "gelu":  # torch.nn.functional.gelu, erf or tanh form
        return F.gelu(args[0], approximate=attrs.get("approximate", "none"))
    if op == "erf":
        return torch.erf(args[0])
    if op == "exp":
        return torch.exp(args[0])
    if op == "rope":
        return _rope(args[0], args[1], args[2], attrs["head_dim"], attrs["seq"])
    raise NotImplementedError(op)


def _arg(env, a):
    t = env[a.tensor]
    if a.cols:
        t = t[:, a.cols[0]:a.cols[1]]
    return t


def run_kernel(spec, env):
    args = {a.name: _arg(env, a) for a in spec.args}
    out = {}
    if spec.kind == "gemm":
        lhs = args["lhs"]
        vals = {g.acc: lhs @ args[g.rhs] for g in spec.gemms}
        if spec.sumsq:
            vals["sumsq"] = (lhs * lhs).sum(-1, keepdim=True)
        for a in spec.args:
            if a.role in ("extra", "const"):
                vals[a.name] = args[a.name]
        for op in spec.epilogue:
            vals[op.name] = _epilogue_op(op.op, [vals[i] for i in op.inputs], op.attrs)
        for o in spec.outputs:
            out[o.tensor] = vals[o.value]
        return out
    a = spec.attrs
    r = {x.role: args[x.name] for x in spec.args}
    if spec.kind == "attention":
        b, s, h, kv, d = a["batch"], a["seq"], a["heads"], a.get("kv_heads", a["heads"]), a["head_dim"]
        q = r["q"].reshape(b, s, h, d).transpose(1, 2)
        k = r["k"].reshape(b, s, kv, d).transpose(1, 2).repeat_interleave(h // kv, 1)
        v = r["v"].reshape(b, s, kv, d).transpose(1, 2).repeat_interleave(h // kv, 1)
        sc = (q @ k.transpose(-1, -2)) * a["scale"]
        if a.get("causal"):
            sc = sc.masked_fill(torch.triu(torch.ones(s, s, dtype=torch.bool), 1), float("-inf"))
        y = (torch.softmax(sc, -1) @ v).transpose(1, 2).reshape(b * s, h * d)
    elif spec.kind == "ssd":
        b, s, h, p, g, n = a["batch"], a["seq"], a["heads"], a["head_dim"], a["ngroups"], a["state_dim"]
        x = r["x"].reshape(b, s, h, p).permute(0, 2, 1, 3)
        B = r["B"].reshape(b, s, g, n).permute(0, 2, 1, 3).repeat_interleave(h // g, 1)
        C = r["C"].reshape(b, s, g, n).permute(0, 2, 1, 3).repeat_interleave(h // g, 1)
        dt = r["dt"].reshape(b, s, h).permute(0, 2, 1)
        dA = dt * r["A"].reshape(1, h, 1)
        y = ssd_chunked(x, dA, dt, B, C, min(256, s)).permute(0, 2, 1, 3).reshape(b * s, h * p)
        if "D" in r:
            y = y + r["x"] * r["D"].reshape(-1).repeat_interleave(p)
        if "z" in r:
            y = y * F.silu(r["z"])
    elif spec.kind == "causal_conv1d":
        x, w = r["x"], r["w"]
        ch, k = w.shape
        xt = x.reshape(a["batch"], a["seq"], ch).transpose(1, 2)
        y = F.conv1d(F.pad(xt, (k - 1, 0)), w.reshape(ch, 1, k), groups=ch).transpose(1, 2).reshape(-1, ch)
        if a.get("act") == "silu":
            y = F.silu(y)
    elif spec.kind == "rmsnorm":
        x = r["x"]
        y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + a["eps"]) * r["gain"].reshape(-1)
    elif spec.kind == "embedding":
        y = r["table"][r["ids"].reshape(-1).long()]
    else:
        raise ValueError(spec.kind)
    out[spec.outputs[0].tensor] = y
    return out


def run_program(program, params, inputs, dtype=torch.float64, allreduce=None):
    """Run every kernel in order; ``allreduce(t)`` (in place) is applied to the
    outputs of kernels marked ``tp_allreduce`` (sharded programs)."""
    if isinstance(inputs, (list, tuple)):
        inputs = dict(zip(program.inputs, inputs))
    env = {}
    for name in program.inputs:
        t = inputs[name]
        shape = program.tensors[name].shape
        env[name] = t.reshape(shape) if t.dtype == torch.int64 else t.reshape(shape).to(dtype)
    for name in program.params:
        v = params[name]
        env[name] = v if v.dtype == torch.int64 else v.to(dtype)
    for spec in program.kernels:
        res = run_kernel(spec, env)
        if spec.attrs.get("tp_allreduce") and allreduce is not None:
            for t in res.values():
                allreduce(t)
        env.update(res)
    return env


def program_outputs(program, params, inputs, dtype=torch.float64, allreduce=None):
    env = run_program(program, params, inputs, dtype, allreduce)
    shapes = program.metadata.get("output_shapes", {})
    return [env[o].reshape(shapes[o]) if o in shapes else env[o] for o in program.outputs]
