"""Canonicalisation: raw OpGraph -> the B200 canonical OpGraph.

Every pass is ``pass(graph) -> rewrites`` and runs in place;
:func:`canonicalize` runs them in order on a copy and, given example
inputs, re-evaluates the graph after each pass that changed it and rejects
a pass that moves any output by more than the tolerance (the reference's
per-pass numeric guard, src/torch_helion/optimizer/passes.py:924-944).

Kept from the reference's pipeline (passes.py:899-921): constant folding,
softplus / rotate-half / RoPE / RMSNorm pattern matching, pushing feature
slices into sibling GEMMs, the RMSNorm row-scale fold into consuming
GEMMs, attention matching, flattening to token-major 2-D, constant
de-duplication.  Changed for B200:

* RoPE stays a ``rope`` op on the token-major tensor (executed on paired
  columns in the producing GEMM's epilogue) instead of the extra W@R GEMM.
* Attention matching also recognises the causal additive mask and grouped
  KV heads (expand+clone of the KV head axis).
* ``match_causal_conv1d`` and ``match_ssd`` are new: the depthwise causal
  conv and the whole Mamba-2 scan (chunked *or* quadratic form, any
  ngroups) become single macro ops; the reference can lower neither
  (it matches only the quadratic form with per-head groups, passes.py:528-610).
* No Loom-only rewrites (unregistered-op expansion, cumsum-as-GEMM,
  32-column padding, materialised rank-1 constants).
"""

from __future__ import annotations

import hashlib
import math
import time
from dataclasses import dataclass
from typing import Callable

import torch

from ..capture.opgraph import OpGraph, OpNode, TensorType
from .evaluate import eval_op, graph_outputs, max_rel_err
from .layout import column_slice, head_merge_fn, match_head_split, trace_layout
from . import param_transforms as pt


class PassError(RuntimeError):
    """The graph holds a construct the B200 lowering cannot express."""


# ------------------------------------------------------------------ helpers
def _convert(g: OpGraph, node: OpNode, op: str, inputs: list[str], attrs: dict | None = None, kind: str = "compute",
             type: TensorType | None = None) -> None:
    g.redefine(node.name, op, inputs, attrs, kind, type)


def _is_const(g: OpGraph, name: str) -> bool:
    return g[name].kind in ("param", "const")


def _strip(g: OpGraph, name: str, ops=("cast", "clone")) -> str:
    """Follow single-input layout nodes in ``ops`` back to their source."""
    while g[name].kind == "layout" and g[name].op in ops and len(g[name].inputs) == 1:
        name = g[name].inputs[0]
    return name


def _const_through_layout(g: OpGraph, name: str) -> str | None:
    """The constant a chain of layout ops reads, if any."""
    while g[name].kind == "layout" and len(g[name].inputs) == 1:
        name = g[name].inputs[0]
    return name if _is_const(g, name) else None


def _matrix_shape(shape: tuple[int, ...]) -> tuple[int, int]:
    """The token-major 2-D shape of a tensor: every axis but the last folded
    into rows (a vector is one row, a scalar a 1 x 1 matrix)."""
    *lead, last = shape or (1,)
    rows = 1
    for extent in lead:
        rows *= extent
    return rows, last


def _ensure_2d(g: OpGraph, name: str) -> str:
    node = g[name]
    if node.type.rank == 2:
        return name
    shape = _matrix_shape(node.type.shape)
    return g.add("view", [name], TensorType(shape, node.type.dtype), {"shape": list(shape)}, kind="layout",
                 origin=f"ensure_2d({name})").name


def _identity_view_users(g: OpGraph, name: str) -> list[tuple[OpNode, OpNode | None]]:
    """Consumers of ``name`` looking through identity reshapes/casts."""
    out: list[tuple[OpNode, OpNode | None]] = []
    for u in g.users(name):
        if u.kind == "layout" and u.op in ("view", "clone", "cast", "expand") and trace_layout(g, u.name).is_identity_reshape():
            out.extend((uu, u) for uu, _ in _identity_view_users(g, u.name))
        else:
            out.append((u, None))
    if name in g.outputs:
        out.append((OpNode("<output>", "output", [name], g[name].type), None))
    return out


def _rebuild_chain(g: OpGraph, chain: list[str], new_base: str, target: OpNode) -> None:
    """Re-apply the layout ops of ``chain`` (base-first) on ``new_base``; the
    last one is written into ``target`` so its users stay valid."""
    prev = new_base
    orig_base_shape = g[g[chain[0]].inputs[0]].type.shape if chain else target.type.shape
    if g[prev].type.shape != orig_base_shape:
        prev = g.add("view", [prev], TensorType(orig_base_shape, g[prev].type.dtype), {"shape": list(orig_base_shape)},
                     kind="layout").name
    if not chain:
        _convert(g, target, "view", [prev], {"shape": list(target.type.shape)}, kind="layout")
        return
    for name in chain[:-1]:
        ln = g[name]
        prev = g.add(ln.op, [prev], ln.type, dict(ln.attrs), kind="layout").name
    last = g[chain[-1]]
    _convert(g, target, last.op, [prev], dict(last.attrs), kind="layout", type=last.type)


# -------------------------------------------------------------------- passes
def fold_constants(g: OpGraph) -> int:
    """Nodes whose inputs are all constant become ``const`` nodes (layout ops
    that would enlarge a constant -- ``expand`` -- are left as views)."""
    n = 0
    for node in list(g):
        if node.kind in ("input", "param", "const") or not node.inputs:
            continue
        if node.op == "expand" or not all(_is_const(g, i) for i in node.inputs):
            continue
        val = eval_op(node.op, [g.value(i) for i in node.inputs], node.attrs)
        val = val.reshape(node.type.shape).to(node.type.torch_dtype).contiguous()
        _convert(g, node, "const", [], {}, kind="const")
        g.params[node.name] = val
        n += 1
    return n


def match_silu(g: OpGraph) -> int:
    """``x * sigmoid(x)`` (the export decomposition of silu) -> ``silu(x)``."""
    n = 0
    for node in list(g):
        if node.op != "mul" or len(node.inputs) != 2:
            continue
        for a, s in (node.inputs, node.inputs[::-1]):
            sn = g[s]
            if sn.op == "sigmoid" and _strip(g, sn.inputs[0]) == _strip(g, a):
                _convert(g, node, "silu", [a])
                n += 1
                break
    return n


def match_softplus(g: OpGraph) -> int:
    """torch's thresholded softplus as export decomposes it --
    ``where(x > t, x, log1p(exp(x)))`` -- becomes ``softplus(x)`` with that
    threshold.  The match starts at ``log1p(exp(x))`` and checks the select
    that consumes it."""
    rewrites = 0
    for soft in [nd for nd in g if nd.op == "log1p"]:
        inner = g[soft.inputs[0]]
        if inner.op != "exp":
            continue
        x = _strip(g, inner.inputs[0])
        for sel in g.users(soft.name):
            if sel.op != "select" or len(sel.inputs) != 3 or sel.inputs[2] != soft.name:
                continue
            test, taken = g[sel.inputs[0]], sel.inputs[1]
            if test.op == "cmp_gt" and "scalar" in test.attrs and _strip(g, test.inputs[0]) == x \
                    and _strip(g, taken) == x:
                _convert(g, sel, "softplus", [test.inputs[0]], {"threshold": float(test.attrs["scalar"])})
                rewrites += 1
    return rewrites


def match_rotate_half(g: OpGraph) -> int:
    n = 0
    for node in list(g):
        if node.op != "cat" or len(node.inputs) != 2 or node.attrs.get("dim") != node.type.rank - 1:
            continue
        a, b = g[node.inputs[0]], g[node.inputs[1]]
        if a.op != "neg" or b.op != "slice":
            continue
        sa = g[a.inputs[0]]
        if sa.op != "slice" or sa.inputs[0] != b.inputs[0]:
            continue
        d = g[sa.inputs[0]].type.shape[-1]
        last = g[sa.inputs[0]].type.rank - 1
        if sa.attrs["dim"] != last or b.attrs["dim"] != last:
            continue
        if (sa.attrs["start"], sa.attrs["end"], b.attrs["start"], b.attrs["end"]) != (d // 2, d, 0, d // 2):
            continue
        _convert(g, node, "rotate_half", [sa.inputs[0]])
        n += 1
    return n


def match_rope(g: OpGraph) -> int:
    """``x*cos + rotate_half(x)*sin`` with constant tables -> ``rope(x, cos, sin)``."""
    n = 0
    for node in list(g):
        if node.op != "add" or len(node.inputs) != 2:
            continue
        m1, m2 = g[node.inputs[0]], g[node.inputs[1]]
        if m1.op != "mul" or m2.op != "mul" or len(m1.inputs) != 2 or len(m2.inputs) != 2:
            continue
        found = None
        for plain, rot in ((m1, m2), (m2, m1)):
            for xi in (0, 1):
                x, cos = plain.inputs[xi], plain.inputs[1 - xi]
                for ri in (0, 1):
                    r, sin = g[rot.inputs[ri]], rot.inputs[1 - ri]
                    if (r.op == "rotate_half" and r.inputs[0] == x and _const_through_layout(g, cos)
                            and _const_through_layout(g, sin)):
                        found = (x, _const_through_layout(g, cos), _const_through_layout(g, sin))
        if found is None:
            continue
        x, cos, sin = found
        _convert(g, node, "rope", [x, cos, sin], {"head_dim": g[x].type.shape[-1]})
        n += 1
    return n


def lower_rope(g: OpGraph) -> int:
    """RoPE on a head-split view -> ``rope`` on the token-major base tensor
    (tables [S, d] in fp32), with the view chain re-applied on top."""
    n = 0
    for node in list(g):
        if node.op != "rope" or g[node.inputs[0]].type.rank == 2:
            continue
        x4, cos, sin = node.inputs
        prov = trace_layout(g, x4)
        dims = match_head_split(prov)
        if dims is None:
            raise PassError(f"rope {node.name}: input is not a head-split view of a token-major tensor")
        s, d = dims["seq"], dims["head_dim"]
        base2d = _ensure_2d(g, prov.base)
        t2 = g[base2d].type
        cv = g.value(cos).float().reshape(-1, d)[:s].contiguous()
        sv = g.value(sin).float().reshape(-1, d)[:s].contiguous()
        if cv.shape[0] != s:
            raise PassError(f"rope {node.name}: table has fewer than {s} positions")
        cc = g.add_const(cv, name=g.fresh_name("rope_cos"))
        sc = g.add_const(sv, name=g.fresh_name("rope_sin"))
        r = g.add("rope", [base2d, cc.name, sc.name], t2, {"head_dim": d, "seq": s, "heads": dims["kv_heads"]},
                  origin=f"lower_rope({node.name})")
        _rebuild_chain(g, prov.chain, r.name, node)
        n += 1
    g.toposort()
    return n


def match_rmsnorm(g: OpGraph) -> int:
    """``x * rsqrt(mean(x^2) + eps) * g`` -> ``rmsnorm(x, g)``."""
    n = 0
    for node in list(g):
        if node.op != "mul" or len(node.inputs) != 2:
            continue
        for inner_n, gain_n in (node.inputs, node.inputs[::-1]):
            gain = _const_through_layout(g, gain_n)
            inner = g[inner_n]
            if gain is None or inner.op != "mul" or len(inner.inputs) != 2:
                continue
            hit = False
            for xn, rn in (inner.inputs, inner.inputs[::-1]):
                r = g[_strip(g, rn)]
                if r.op != "rsqrt":
                    continue
                add = g[_strip(g, r.inputs[0])]
                if add.op != "add" or "scalar" not in add.attrs:
                    continue
                mean = g[_strip(g, add.inputs[0])]
                if mean.op != "row_mean":
                    continue
                sq = g[_strip(g, mean.inputs[0])]
                src = _strip(g, xn)
                ok = ((sq.op == "powf" and sq.attrs.get("scalar") == 2 and _strip(g, sq.inputs[0]) == src)
                      or (sq.op == "square" and _strip(g, sq.inputs[0]) == src)
                      or (sq.op == "mul" and len(sq.inputs) == 2 and all(_strip(g, i) == src for i in sq.inputs)))
                if not ok:
                    continue
                _convert(g, node, "rmsnorm", [xn, gain], {"eps": float(add.attrs["scalar"])})
                n += 1
                hit = True
                break
            if hit:
                break
    return n


def _producing_gemm(g: OpGraph, name: str) -> OpNode | None:
    """The constant-RHS matmul whose columns ``name`` shows unchanged: the
    value may sit behind identity reshapes / copies / casts that keep the
    column axis, nothing else."""
    cols = g[name].type.shape[-1]
    hops = [g[name]]
    while hops[-1].kind == "layout":
        node = hops[-1]
        keeps_cols = (node.op in ("view", "clone", "cast") and len(node.inputs) == 1
                      and node.type.shape[-1] == cols and trace_layout(g, node.name).is_identity_reshape())
        if not keeps_cols:
            return None
        hops.append(g[node.inputs[0]])
    root = hops[-1]
    is_gemm = root.op == "matmul" and root.type.shape[-1] == cols
    return root if is_gemm and _const_through_layout(g, root.inputs[1]) else None


def push_slice_into_gemm(g: OpGraph) -> int:
    """``slice(a @ W, cols)`` -> ``a @ W[:, cols]``: split projections become
    sibling GEMMs sharing their LHS (reference passes.py:390-416)."""
    n = 0
    while True:
        progressed = False
        for node in list(g):
            if node.op != "slice" or node.attrs.get("dim") != g[node.inputs[0]].type.rank - 1:
                continue
            src = _producing_gemm(g, node.inputs[0])
            if src is None:
                continue
            lo, hi = node.attrs["start"], node.attrs["end"]
            w = _const_through_layout(g, src.inputs[1])
            wfull = _materialize(g, src.inputs[1])
            wc = g.add_const(wfull[:, lo:hi].contiguous().to(g[w].type.torch_dtype), name=g.fresh_name(w + "_cols"))
            _convert(g, node, "matmul", [src.inputs[0], wc.name], {}, type=node.type)
            n += 1
            progressed = True
        if not progressed:
            break
    g.toposort()
    return n


def _materialize(g: OpGraph, name: str) -> torch.Tensor:
    """Value of a constant seen through a chain of layout ops."""
    node = g[name]
    if _is_const(g, name):
        return g.value(name)
    if node.kind == "layout" and len(node.inputs) == 1:
        return eval_op(node.op, [_materialize(g, node.inputs[0])], node.attrs).to(node.type.torch_dtype)
    raise PassError(f"{name} is not a constant")


def _row_scale(g: OpGraph, x2d: str, eps: float, origin: str) -> str:
    """``(row_sumsq(x)/K + eps) ** -0.5`` as a [T, 1] column (passes.py:347-354)."""
    t, k = g[x2d].type.shape
    col = TensorType((t, 1), g[x2d].type.dtype)
    ss = g.add("row_sumsq", [x2d], col, origin=origin)
    m = g.add("mul", [ss.name], col, {"scalar": 1.0 / k})
    a = g.add("add", [m.name], col, {"scalar": eps})
    return g.add("powf", [a.name], col, {"scalar": -0.5}, origin=origin).name


def lower_rmsnorm(g: OpGraph) -> int:
    """RMSNorm feeding only constant-RHS GEMMs: fold the gain into the weights
    and the row scale into the GEMM epilogue (reference passes.py:252-285).
    Any other RMSNorm stays a 2-D ``rmsnorm`` op (the B200 norm kernel)."""
    n = 0
    for node in list(g):
        if node.op != "rmsnorm" or node.attrs.get("lowered"):
            continue
        x, gain = node.inputs
        eps = node.attrs["eps"]
        users = _identity_view_users(g, node.name)
        gemm_users = [(u, via) for u, via in users
                      if u.op == "matmul" and _const_through_layout(g, u.inputs[1])
                      and u.inputs[0] == (via.name if via else node.name)]
        x2d = _ensure_2d(g, x)
        gval = _materialize(g, gain).reshape(-1)
        if users and len(gemm_users) == len(users):
            r = _row_scale(g, x2d, eps, f"lower_rmsnorm({node.name})")
            for mm, _via in gemm_users:
                w = _materialize(g, mm.inputs[1])
                wg = g.add_const(pt.fold_gain_into_weight(gval, w), name=g.fresh_name(mm.inputs[1] + "_norm"))
                flat = TensorType(_matrix_shape(mm.type.shape), mm.type.dtype)
                new_mm = g.add("matmul", [x2d, wg.name], flat, origin=f"lower_rmsnorm({mm.name})")
                bc = g.add("broadcast", [r], flat, {"dim": 1, "shape": list(flat.shape)})
                sc = g.add("mul", [new_mm.name, bc.name], flat)
                _convert(g, mm, "view", [sc.name], {"shape": list(mm.type.shape)}, kind="layout")
        else:
            gc = g.add_const(gval.float().contiguous(), name=g.fresh_name(gain + "_f32"))
            t2 = TensorType(_matrix_shape(node.type.shape), node.type.dtype)
            rn = g.add("rmsnorm", [x2d, gc.name], t2, {"eps": eps, "lowered": True}, origin=f"rmsnorm({node.name})")
            _convert(g, node, "view", [rn.name], {"shape": list(node.type.shape)}, kind="layout")
        n += 1
    g.toposort()
    return n


def _causal_mask_value(v: torch.Tensor, s: int) -> bool:
    """True when ``v`` broadcasts to an [s, s] additive causal mask."""
    v = v.float()
    if v.numel() != s * s:
        return False
    m = v.reshape(s, s)
    upper = torch.triu(torch.ones(s, s, dtype=torch.bool), 1)
    return bool((m[~upper] == 0).all() and torch.isneginf(m[upper]).all())


def match_attention(g: OpGraph) -> int:
    """bmm -> [scale] -> [+ causal mask] -> softmax -> bmm on head-split views
    -> ``attention(q, k, v)`` (reference passes.py:419-471, extended with the
    causal mask and grouped KV heads)."""
    n = 0
    for sm in list(g):
        if sm.op != "softmax":
            continue
        s = g[_strip(g, sm.inputs[0])]
        causal = False
        if s.op == "add" and len(s.inputs) == 2:
            for other, m in (s.inputs, s.inputs[::-1]):
                c = _const_through_layout(g, m)
                if c is not None and _causal_mask_value(_materialize(g, m), s.type.shape[-1]):
                    causal = True
                    s = g[_strip(g, other)]
                    break
        scale = 1.0
        if s.op == "mul" and "scalar" in s.attrs:
            scale = float(s.attrs["scalar"])
            s = g[_strip(g, s.inputs[0])]
        prov_s = trace_layout(g, s.name)
        bmm1 = g[prov_s.base]
        if bmm1.op != "batch_matmul" or not prov_s.is_identity_reshape():
            continue
        dq = match_head_split(trace_layout(g, bmm1.inputs[0]))
        dk = match_head_split(trace_layout(g, bmm1.inputs[1]), transpose_last=True)
        if dq is None or dk is None or dq["kv_heads"] != dq["heads"]:
            continue
        key = lambda d: (d["batch"], d["seq"], d["heads"], d["head_dim"])
        if key(dq) != key(dk):
            continue
        cons = [u for u, _ in _identity_view_users(g, sm.name)]
        if len(cons) != 1 or cons[0].op != "batch_matmul":
            continue
        bmm2 = cons[0]
        prov_p = trace_layout(g, bmm2.inputs[0])
        if prov_p.base != sm.name or not prov_p.is_identity_reshape():
            continue
        dv = match_head_split(trace_layout(g, bmm2.inputs[1]))
        if dv is None or key(dv) != key(dq) or dv["kv_heads"] != dk["kv_heads"]:
            continue
        b, sq, h, d = key(dq)
        merge = head_merge_fn(b, sq, h, d)
        final, cur = None, bmm2
        while True:
            users = g.users(cur.name)
            if len(users) != 1 or users[0].kind != "layout":
                break
            cur = users[0]
            prov = trace_layout(g, cur.name)
            if prov.base == bmm2.name and prov.numel == b * sq * h * d and len(prov.shape) >= 2 \
                    and prov.shape[-1] == h * d:
                flat = prov  # token-major candidate: [B, S, H*d] or [T, H*d]
                p = flat.probes()
                rows = p[:, :-1]
                t = rows[:, 0] * sq + rows[:, 1] if rows.shape[1] == 2 else rows[:, 0]
                if torch.equal(flat.to_base(p), merge(torch.stack((t, p[:, -1]), 1))):
                    final = cur
                    break
        if final is None:
            continue
        ins = [_ensure_2d(g, trace_layout(g, bmm1.inputs[0]).base), _ensure_2d(g, trace_layout(g, bmm1.inputs[1]).base),
               _ensure_2d(g, trace_layout(g, bmm2.inputs[1]).base)]
        _convert(g, final, "attention", ins, {"batch": b, "seq": sq, "heads": h, "kv_heads": dk["kv_heads"], "head_dim": d,
                                           "scale": scale, "causal": causal},
                 type=TensorType((b * sq, h * d), final.type.dtype))
        n += 1
    g.toposort()
    return n


def match_causal_conv1d(g: OpGraph) -> int:
    """``permute -> pad(k-1, 0) -> depthwise conv1d -> permute`` on a
    token-major [B, S, C] tensor -> ``causal_conv1d(x2d, w[C, k])``
    (models/mamba.py:278-283)."""
    n = 0
    for cv in list(g):
        if cv.op != "conv1d" or len(cv.inputs) != 2:
            continue
        a = cv.attrs
        pad = g[cv.inputs[0]]
        b, ch, s_out = cv.type.shape
        wname = _const_through_layout(g, cv.inputs[1])
        if (a["groups"] != ch or a["stride"] != [1] or a["padding"] != [0] or a["dilation"] != [1] or wname is None
                or pad.op != "pad" or pad.attrs.get("value", 0.0) != 0.0):
            continue
        w = _materialize(g, cv.inputs[1])
        k = w.shape[-1]
        if pad.attrs["pad"] != [k - 1, 0] or w.numel() != ch * k:
            continue
        prov_in = trace_layout(g, pad.inputs[0])
        s = prov_in.shape[-1]
        if prov_in.shape != (b, ch, s) or math.prod(prov_in.base_shape) != b * s * ch:
            continue
        if not prov_in.matches(lambda c: (c[:, 0] * s + c[:, 2]) * ch + c[:, 1]):
            continue
        # the token-major view of the conv output: [B, S, C] reading conv[b, c, s]
        final, cur = None, cv
        while True:
            users = g.users(cur.name)
            if len(users) != 1 or users[0].kind != "layout":
                break
            cur = users[0]
            prov = trace_layout(g, cur.name)
            if prov.base == cv.name and prov.shape in ((b, s, ch), (b * s, ch)):
                rowcol = lambda c: (c[:, 0] // s, c[:, 0] % s, c[:, 1]) if c.shape[1] == 2 else (c[:, 0], c[:, 1], c[:, 2])
                if prov.matches(lambda c: (lambda bi, si, ci: (bi * ch + ci) * s + si)(*rowcol(c))):
                    final = cur
                    break
        if final is None:
            continue
        x2d = _ensure_2d(g, prov_in.base)
        wc = g.add_const(w.reshape(ch, k).float().contiguous(), name=g.fresh_name(wname + "_f32"))
        node = g.add("causal_conv1d", [x2d, wc.name], TensorType((b * s, ch), final.type.dtype),
                     {"batch": b, "seq": s, "width": k, "act": None}, origin=f"match_causal_conv1d({cv.name})")
        _rebuild_chain(g, [], node.name, final)
        n += 1
    g.toposort()
    return n


def _token_major(g: OpGraph) -> tuple[int, int] | None:
    """(batch, seq) of the graph's first input ([B, S, ...] or [B, S] ids)."""
    if not g.inputs:
        return None
    sh = g[g.inputs[0]].type.shape
    return (sh[0], sh[1]) if len(sh) >= 2 else None


def match_ssd(g: OpGraph) -> int:
    """The Mamba-2 scan -> one ``ssd`` op, from either evaluation form.

    The scan region is the connected set of non-token-major nodes around a
    ``batch_matmul`` (no softmax: attention is matched first).  Its inputs
    are token-major tensors and constants; its single output is the
    token-major view of ``y + D*x``.  Roles follow from the math:
    C and B are the left/right operands of the Gram product C B^T, x is the
    input as wide as the output, dt the remaining per-head input, A and D
    the per-head constants multiplied with dt and x.  The pass's numeric
    check (``canonicalize``) confirms the match end to end."""
    bs = _token_major(g)
    if bs is None:
        return 0
    B_, S_ = bs
    T = B_ * S_

    def tm(node: OpNode) -> bool:
        sh = node.type.shape
        return (len(sh) == 3 and sh[:2] == (B_, S_)) or (len(sh) == 2 and sh[0] == T)

    umap = g.user_map()
    n = 0
    seen: set[str] = set()
    for seed in list(g):
        if seed.name not in g.nodes or seed.op != "batch_matmul" or seed.name in seen:
            continue
        region: set[str] = set()
        inputs: set[str] = set()
        outputs: set[str] = set()
        stack = [seed.name]
        while stack:
            nm = stack.pop()
            if nm in region:
                continue
            region.add(nm)
            for i in g[nm].inputs:
                if _is_const(g, i) or tm(g[i]):
                    inputs.add(i)
                elif i not in region:
                    stack.append(i)
            for u in umap.get(nm, []):
                if tm(g[u]):
                    outputs.add(u)
                elif u not in region:
                    stack.append(u)
        seen |= region
        ops = {g[r].op for r in region}
        if "softmax" in ops or "exp" not in ops or len(outputs) != 1:
            continue
        out = g[next(iter(outputs))]
        acts = [i for i in inputs if not _is_const(g, i)]
        consts = [i for i in inputs if _is_const(g, i)]

        def source(nm: str) -> str | None:
            while nm not in inputs:
                node = g[nm]
                if node.kind != "layout" or len(node.inputs) != 1:
                    return None
                nm = node.inputs[0]
            return nm

        gram = [(source(g[r].inputs[0]), source(g[r].inputs[1])) for r in region if g[r].op == "batch_matmul"]
        gram = [(c, b) for c, b in gram if c in acts and b in acts and c != b]
        if len(gram) != 1:
            continue
        Cn, Bn = gram[0]
        width = out.type.shape[-1]
        xs = [a for a in acts if a not in (Cn, Bn) and g[a].type.shape[-1] == width]
        dts = [a for a in acts if a not in (Cn, Bn) and a not in xs]
        if len(xs) != 1 or len(dts) != 1 or len(acts) != 4:
            continue
        xn, dtn = xs[0], dts[0]
        H = g[dtn].type.shape[-1]
        if width % H:
            continue
        P = width // H
        G, N = 1, g[Bn].type.shape[-1]
        for u in umap.get(Bn, []):
            un = g[u]
            if un.op == "view" and un.name in region and un.type.rank >= 4:
                G, N = un.type.shape[-2], un.type.shape[-1]
                break
        if G * N != g[Bn].type.shape[-1] or H % G:
            continue
        A = D = None
        for c in consts:
            if g[c].type.numel != H:
                continue
            for u in umap.get(c, []):
                un = g[u]
                if un.op != "mul" or un.name not in region or len(un.inputs) != 2:
                    continue
                other = un.inputs[1] if un.inputs[0] == c else un.inputs[0]
                src = source(other)
                if src == dtn:
                    A = c
                elif src == xn:
                    D = c
        if A is None:
            continue
        # the model's chunk length (its [l, l] masks), kept as a hint: the
        # scan's value does not depend on how the sequence is chunked
        squares = [g[c].type.shape[0] for c in consts
                   if g[c].type.rank == 2 and g[c].type.shape[0] == g[c].type.shape[1] and g[c].type.shape[0] < S_]
        chunk = max(squares) if squares else 256
        ins = [_ensure_2d(g, xn), _ensure_2d(g, dtn)]
        ac = g.add_const(g.value(A).float().reshape(H).contiguous(), name=g.fresh_name("ssd_A"))
        ins += [ac.name, _ensure_2d(g, Bn), _ensure_2d(g, Cn)]
        if D is not None:
            ins.append(g.add_const(g.value(D).float().reshape(H).contiguous(), name=g.fresh_name("ssd_D")).name)
        node = g.add("ssd", ins, TensorType((T, width), out.type.dtype),
                     {"batch": B_, "seq": S_, "heads": H, "head_dim": P, "ngroups": G, "state_dim": N, "chunk": chunk,
                      "has_D": D is not None, "gate": False}, origin=f"match_ssd({out.name})")
        _rebuild_chain(g, [], node.name, out)
        umap = g.user_map()
        n += 1
    g.toposort()
    return n


def flatten_to_2d(g: OpGraph) -> int:
    """Remove identity reshapes; keep column slices of 2-D tensors (free views
    for the kernels); give every activation a token-major 2-D type."""
    n = 0
    identity: list[tuple[str, str]] = []
    for node in list(g):
        if node.kind != "layout":
            continue
        prov = trace_layout(g, node.name)
        if node.op in ("view", "clone", "expand", "cast", "permute", "slice") and prov.is_identity_reshape():
            identity.append((node.name, prov.base))
            continue
        cs = column_slice(prov) if node.op in ("slice", "view", "clone", "cast") else None
        if cs is not None:
            base2d = _ensure_2d(g, prov.base)
            _convert(g, node, "slice", [base2d], {"dim": 1, "start": cs[0], "end": cs[1]}, kind="layout",
                     type=TensorType(_matrix_shape(node.type.shape), node.type.dtype))
            continue
        raise PassError(f"layout op {node.name} ({node.op}) survived canonicalisation: {node.type} is a "
                        f"reshape/permute view of {prov.base} {g[prov.base].type} via {prov.chain}")
    for name, base in identity:
        g.replace_all_uses(name, base)
        n += 1
    g.dce()
    shapes = {}
    for node in g:
        if node.kind in ("param", "const"):
            continue
        if node.kind == "input":
            shapes[node.name] = list(node.type.shape)
        if node.op == "broadcast":
            node.attrs["shape"] = list(_matrix_shape(tuple(node.attrs["shape"])))
        if node.kind == "input" and node.type.dtype == "int64":
            node.type = TensorType((math.prod(node.type.shape), 1), "int64")
            continue
        node.type = TensorType(_matrix_shape(node.type.shape), node.type.dtype)
    floats = [g[i].type.dtype for i in g.inputs if g[i].type.dtype != "int64"]
    if floats:
        act = floats[0]
    else:
        emb = [g[nd.inputs[1]].type.dtype for nd in g if nd.op == "embedding"]
        act = emb[0] if emb else "float32"
    for node in g:
        if node.kind in ("param", "const", "input"):
            continue
        node.type = TensorType(node.type.shape, act)
    # views created above (ensure_2d on a 3-D base) are identities now
    for node in list(g):
        if node.kind == "layout" and node.op in ("view", "clone", "cast") and g[node.inputs[0]].type.shape == node.type.shape:
            g.replace_all_uses(node.name, node.inputs[0])
            n += 1
    g.dce()
    g.metadata.setdefault("input_shapes", shapes)
    g.metadata.setdefault("output_shapes", g.metadata.get("output_shapes_raw", {}))
    g.metadata["dtype"] = act
    g.toposort()
    return n


def fuse_conv_activation(g: OpGraph) -> int:
    n = 0
    for node in list(g):
        if node.op != "silu":
            continue
        src = g[node.inputs[0]]
        if src.op == "causal_conv1d" and src.attrs.get("act") is None and g.num_uses(src.name) == 1:
            _convert(g, node, "causal_conv1d", list(src.inputs), {**src.attrs, "act": "silu"})
            g.dce()
            n += 1
    return n


def fuse_ssd_gate(g: OpGraph) -> int:
    """``ssd(...) * silu(z)`` -> ``ssd(..., z)`` with the gate fused."""
    n = 0
    for node in list(g):
        if node.op != "mul" or len(node.inputs) != 2:
            continue
        for a, b in (node.inputs, node.inputs[::-1]):
            s, z = g[a], g[b]
            if s.op == "ssd" and not s.attrs.get("gate") and z.op == "silu" and g.num_uses(s.name) == 1:
                _convert(g, node, "ssd", list(s.inputs) + [z.inputs[0]], {**s.attrs, "gate": True})
                g.dce()
                n += 1
                break
    g.toposort()
    return n


def dedupe_constants(g: OpGraph) -> int:
    """Constants with identical type and bytes are merged into the first one
    (up to 4 Mi elements; larger tables are left alone).  Candidates are
    bucketed by a BLAKE2 digest of their bytes and confirmed with
    ``torch.equal``, so dtypes without a numpy view (bf16) work too."""
    buckets: dict[tuple, list[str]] = {}
    merged = 0
    for node in [nd for nd in g if nd.kind == "const"]:
        value = g.value(node.name)
        if value.numel() >= (1 << 22):
            continue
        raw = value.detach().contiguous().reshape(-1).view(torch.uint8)
        digest = hashlib.blake2b(raw.numpy().tobytes(), digest_size=16).digest()
        key = (tuple(node.type.shape), node.type.dtype, digest)
        twin = next((k for k in buckets.get(key, ()) if torch.equal(g.value(k), value)), None)
        if twin is None:
            buckets.setdefault(key, []).append(node.name)
        else:
            g.replace_all_uses(node.name, twin)
            merged += 1
    return merged


def cleanup(g: OpGraph) -> int:
    n = g.dce()
    g.toposort()
    return n


@dataclass(frozen=True)
class Pass:
    """One canonicalisation step: ``run(graph) -> rewrites``.  ``stage`` groups
    the steps the way the B200 lowering needs them: pattern matches on the raw
    graph, lowerings to B200 macro ops, the 2-D flattening, and tidy-ups."""

    name: str
    run: Callable[[OpGraph], int]
    stage: str


PIPELINE: tuple[Pass, ...] = (
    Pass("fold_constants", fold_constants, "match"),
    Pass("match_silu", match_silu, "match"),
    Pass("match_softplus", match_softplus, "match"),
    Pass("match_rotate_half", match_rotate_half, "match"),
    Pass("match_rope", match_rope, "match"),
    Pass("lower_rope", lower_rope, "lower"),
    Pass("match_rmsnorm", match_rmsnorm, "match"),
    Pass("push_slice_into_gemm", push_slice_into_gemm, "lower"),
    Pass("lower_rmsnorm", lower_rmsnorm, "lower"),
    Pass("match_attention", match_attention, "match"),
    Pass("match_causal_conv1d", match_causal_conv1d, "match"),
    Pass("match_ssd", match_ssd, "match"),
    Pass("fold_constants_2", fold_constants, "tidy"),
    Pass("cleanup_1", cleanup, "tidy"),
    Pass("flatten_to_2d", flatten_to_2d, "layout"),
    Pass("fuse_conv_activation", fuse_conv_activation, "lower"),
    Pass("fuse_ssd_gate", fuse_ssd_gate, "lower"),
    Pass("dedupe_constants", dedupe_constants, "tidy"),
    Pass("cleanup_2", cleanup, "tidy"),
)
# the reference's name for the pass list: (name, function) pairs
PASSES: list[tuple[str, Callable[[OpGraph], int]]] = [(p.name, p.run) for p in PIPELINE]


class _Checker:
    """Evaluates the graph on the verification inputs and compares its outputs
    with those of the raw graph (the reference's error metric, max |a-b| /
    max |b|)."""

    def __init__(self, raw: OpGraph, inputs: list[torch.Tensor] | None, tolerance: float) -> None:
        self.inputs, self.tolerance = inputs, tolerance
        self.want = graph_outputs(raw, inputs) if inputs is not None else None

    def error(self, g: OpGraph) -> float | None:
        if self.want is None:
            return None
        got = graph_outputs(g, self.inputs)
        return max(max_rel_err(a.reshape(-1), b.reshape(-1)) for a, b in zip(got, self.want))


def canonicalize(graph: OpGraph, verify_inputs: list[torch.Tensor] | None = None,
                 tolerance: float = 2e-2) -> tuple[OpGraph, list[dict]]:
    """Run :data:`PIPELINE` on a copy of ``graph``.  With ``verify_inputs``
    every step that rewrote something is checked numerically against the raw
    graph and a step that moves the outputs by more than ``tolerance`` raises
    :class:`PassError`.  Returns the canonical graph and the per-step log."""
    g = graph.copy()
    out_shapes = [list(g[o].type.shape) for o in g.outputs]
    g.metadata["output_shapes_raw"] = dict(zip(g.outputs, out_shapes))
    checker = _Checker(g, verify_inputs, tolerance)
    log: list[dict] = []
    for step in PIPELINE:
        t0 = time.perf_counter()
        rewrites = step.run(g)
        record = {"pass": step.name, "stage": step.stage, "rewrites": rewrites, "nodes": len(g),
                  "seconds": round(time.perf_counter() - t0, 4)}
        if rewrites:
            err = checker.error(g)
            if err is not None:
                record["max_rel_err"] = err
                if not err <= tolerance:
                    raise PassError(f"pass {step.name} changed the numerics (max rel err {err:.3e} > {tolerance})")
        log.append(record)
    # rewrites may rename the outputs; their shapes are kept by position
    g.metadata["output_shapes"] = dict(zip(g.outputs, out_shapes))
    return g, log
