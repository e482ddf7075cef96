"""Core-ATen FX graph -> raw OpGraph.

A literal translation, as in the reference (src/torch_helion/capture/
fx_to_opgraph.py:80-121): one OpGraph node per ATen node with the same
shape, layout ops kept as ``layout`` nodes, parameters/buffers/lifted
constants emitted with their values, and every semantic rewrite left to the
optimizer.  Handlers added for the B200 workloads: ``constant_pad_nd``,
``convolution`` (Mamba's depthwise causal conv) and ``embedding``.
Unsupported ops raise :class:`UnsupportedOpError`.
"""

from __future__ import annotations

from typing import Any, Callable

import torch
from torch.fx import Node

from .fx_capture import CapturedFx
from .opgraph import OpGraph, OpNode, TensorType


class UnsupportedOpError(NotImplementedError):
    """An ATen op has no OpGraph mapping."""


_HANDLERS: dict[str, Callable[["_Converter", Node], OpNode]] = {}


def _on(*targets: str):
    def deco(fn):
        for t in targets:
            _HANDLERS[t] = fn
        return fn

    return deco


def _tt(node: Node) -> TensorType:
    val = node.meta.get("val")
    if not isinstance(val, torch.Tensor):
        raise UnsupportedOpError(f"{node.name}: non-tensor value {type(val).__name__}")
    return TensorType(tuple(int(s) for s in val.shape), str(val.dtype).replace("torch.", ""))


def _dim(d: int, rank: int) -> int:
    return d + rank if d < 0 else d


class _Converter:
    def __init__(self, captured: CapturedFx) -> None:
        self.captured = captured
        self.ep = captured.exported
        self.gm = captured.graph_module
        self.graph = OpGraph("model")
        self.names: dict[str, str] = {}
        self.splits: dict[str, tuple[str, list[int], int]] = {}

    def src(self, arg: Any) -> str:
        if isinstance(arg, Node):
            return self.names[arg.name]
        raise UnsupportedOpError(f"expected a tensor operand, got {arg!r}")

    def emit(self, node: Node, op: str, inputs: list[str], attrs: dict | None = None, kind: str = "compute") -> OpNode:
        out = self.graph.add(op, inputs, _tt(node), attrs=attrs, kind=kind, name=node.name, origin=str(node.target))
        self.names[node.name] = out.name
        return out

    def binary(self, node: Node, op: str) -> OpNode:
        a, b = node.args[0], node.args[1]
        if isinstance(a, Node) and isinstance(b, Node):
            return self.emit(node, op, [self.src(a), self.src(b)])
        if isinstance(a, Node):
            return self.emit(node, op, [self.src(a)], {"scalar": float(b)})
        return self.emit(node, op, [self.src(b)], {"scalar": float(a), "scalar_first": True})

    def value_node(self, node: Node, kind: str, pname: str, value: torch.Tensor | None, t: TensorType) -> None:
        name = pname.replace(".", "_")
        val = value.detach().clone() if value is not None else None
        out = self.graph.add(kind, [], t, kind=kind, name=name, origin=node.name, value=val)
        self.names[node.name] = out.name

    def run(self) -> OpGraph:
        sig = self.ep.graph_signature
        params = dict(self.ep.state_dict)
        consts = getattr(self.ep, "constants", {}) or {}
        lifted = getattr(sig, "inputs_to_lifted_tensor_constants", {}) or {}
        for node in self.gm.graph.nodes:
            if node.op == "placeholder":
                t = _tt(node)
                if node.name in sig.inputs_to_parameters:
                    pn = sig.inputs_to_parameters[node.name]
                    self.value_node(node, "param", pn, params[pn], t)
                elif node.name in sig.inputs_to_buffers:
                    bn = sig.inputs_to_buffers[node.name]
                    self.value_node(node, "param", bn, params.get(bn, consts.get(bn)), t)
                elif node.name in lifted:
                    cn = lifted[node.name]
                    self.value_node(node, "const", cn, consts[cn], t)
                else:
                    self.value_node(node, "input", node.name, None, t)
            elif node.op == "call_function":
                key = str(node.target)
                if key == "aten.split_with_sizes.default":
                    src = node.args[0]
                    rank = len(_tt(src).shape)
                    dim = _dim(int(node.args[2]) if len(node.args) > 2 else 0, rank)
                    self.splits[node.name] = (self.src(src), [int(v) for v in node.args[1]], dim)
                    continue
                fn = _HANDLERS.get(key)
                if fn is None:
                    raise UnsupportedOpError(f"no OpGraph mapping for {key} (node {node.name})")
                fn(self, node)
            elif node.op == "output":
                outs = node.args[0]
                outs = outs if isinstance(outs, (tuple, list)) else (outs,)
                self.graph.outputs = [self.src(o) for o in outs]
            else:
                raise UnsupportedOpError(f"unsupported fx node kind {node.op} ({node.target})")
        self.graph.metadata["fx_op_histogram"] = self.captured.op_histogram()
        return self.graph


# ------------------------------------------------------------------ handlers
for _t, _o in {"aten.add.Tensor": "add", "aten.sub.Tensor": "sub", "aten.mul.Tensor": "mul", "aten.div.Tensor": "div",
               "aten.maximum.default": "max"}.items():
    _HANDLERS[_t] = (lambda op: (lambda c, n: c.binary(n, op)))(_o)


@_on("aten.pow.Tensor_Scalar")
def _pow_s(c, n):
    return c.emit(n, "powf", [c.src(n.args[0])], {"scalar": float(n.args[1])})


@_on("aten.pow.Tensor_Tensor")
def _pow_t(c, n):
    return c.emit(n, "powf", [c.src(n.args[0]), c.src(n.args[1])])


for _t, _o in {"aten.exp.default": "exp", "aten.log.default": "log", "aten.neg.default": "neg",
               "aten.rsqrt.default": "rsqrt", "aten.sqrt.default": "sqrt", "aten.sigmoid.default": "sigmoid",
               "aten.silu.default": "silu", "aten.tanh.default": "tanh", "aten.square.default": "square",
               "aten.log1p.default": "log1p"}.items():
    _HANDLERS[_t] = (lambda op: (lambda c, n: c.emit(n, op, [c.src(n.args[0])])))(_o)


@_on("aten.mean.dim", "aten.sum.dim_IntList", "aten.amax.default")
def _reduce(c, n):
    x = n.args[0]
    dims = n.args[1] if len(n.args) > 1 else None
    keep = bool(n.args[2]) if len(n.args) > 2 else bool(n.kwargs.get("keepdim", False))
    rank = len(_tt(x).shape)
    dims = [dims] if isinstance(dims, int) else list(dims or [])
    dims = [_dim(int(d), rank) for d in dims]
    if dims != [rank - 1]:
        raise UnsupportedOpError(f"{n.name}: only last-axis reductions are supported (dims={dims})")
    op = {"aten.mean.dim": "row_mean", "aten.sum.dim_IntList": "row_sum", "aten.amax.default": "row_max"}[str(n.target)]
    return c.emit(n, op, [c.src(x)], {"keepdim": keep})


@_on("aten._softmax.default", "aten.softmax.int")
def _softmax(c, n):
    rank = len(_tt(n.args[0]).shape)
    if _dim(int(n.args[1]), rank) != rank - 1:
        raise UnsupportedOpError(f"{n.name}: softmax only over the last axis")
    return c.emit(n, "softmax", [c.src(n.args[0])])


@_on("aten.mm.default")
def _mm(c, n):
    return c.emit(n, "matmul", [c.src(n.args[0]), c.src(n.args[1])])


@_on("aten.bmm.default")
def _bmm(c, n):
    return c.emit(n, "batch_matmul", [c.src(n.args[0]), c.src(n.args[1])])


@_on("aten.addmm.default")
def _addmm(c, n):
    bias, a, b = n.args[:3]
    mm = c.graph.add("matmul", [c.src(a), c.src(b)], _tt(n), name=n.name + "_mm", origin="aten.addmm")
    return c.emit(n, "add", [mm.name, c.src(bias)])


@_on("aten.permute.default")
def _permute(c, n):
    return c.emit(n, "permute", [c.src(n.args[0])], {"dims": [int(d) for d in n.args[1]]}, kind="layout")


@_on("aten.transpose.int")
def _transpose(c, n):
    rank = len(_tt(n.args[0]).shape)
    d0, d1 = _dim(int(n.args[1]), rank), _dim(int(n.args[2]), rank)
    dims = list(range(rank))
    dims[d0], dims[d1] = dims[d1], dims[d0]
    return c.emit(n, "permute", [c.src(n.args[0])], {"dims": dims}, kind="layout")


@_on("aten.t.default")
def _t(c, n):
    return c.emit(n, "permute", [c.src(n.args[0])], {"dims": [1, 0]}, kind="layout")


@_on("aten.view.default", "aten.reshape.default", "aten._unsafe_view.default", "aten.unsqueeze.default",
     "aten.squeeze.dim", "aten.squeeze.default", "aten.squeeze.dims")
def _view(c, n):
    return c.emit(n, "view", [c.src(n.args[0])], {"shape": list(_tt(n).shape)}, kind="layout")


@_on("aten.expand.default")
def _expand(c, n):
    return c.emit(n, "expand", [c.src(n.args[0])], {"shape": list(_tt(n).shape)}, kind="layout")


@_on("aten.clone.default", "aten.contiguous.default", "aten.alias.default", "aten.detach.default")
def _clone(c, n):
    return c.emit(n, "clone", [c.src(n.args[0])], kind="layout")


@_on("aten._to_copy.default", "aten.to.dtype")
def _cast(c, n):
    return c.emit(n, "cast", [c.src(n.args[0])], {"dtype": _tt(n).dtype}, kind="layout")


@_on("aten.slice.Tensor")
def _slice(c, n):
    x = n.args[0]
    rank = len(_tt(x).shape)
    dim = _dim(int(n.args[1]) if len(n.args) > 1 else 0, rank)
    size = _tt(x).shape[dim]
    start = int(n.args[2]) if len(n.args) > 2 and n.args[2] is not None else 0
    end = int(n.args[3]) if len(n.args) > 3 and n.args[3] is not None else size
    step = int(n.args[4]) if len(n.args) > 4 else 1
    if step != 1:
        raise UnsupportedOpError(f"{n.name}: strided slice")
    start = max(0, start + size if start < 0 else start)
    end = min(size, end + size if end < 0 else end)
    return c.emit(n, "slice", [c.src(x)], {"dim": dim, "start": start, "end": end}, kind="layout")


@_on("<built-in function getitem>")
def _getitem(c, n):
    src, idx = n.args[0], int(n.args[1])
    if not isinstance(src, Node) or src.name not in c.splits:
        raise UnsupportedOpError(f"{n.name}: getitem on something other than a tensor split")
    base, sizes, dim = c.splits[src.name]
    start = sum(sizes[:idx])
    return c.emit(n, "slice", [base], {"dim": dim, "start": start, "end": start + sizes[idx]}, kind="layout")


@_on("aten.cumsum.default")
def _cumsum(c, n):
    rank = len(_tt(n.args[0]).shape)
    if _dim(int(n.args[1]) if len(n.args) > 1 else -1, rank) != rank - 1:
        raise UnsupportedOpError(f"{n.name}: only last-axis cumsum")
    return c.emit(n, "row_cumsum", [c.src(n.args[0])])


@_on("aten.gt.Scalar")
def _gt(c, n):
    return c.emit(n, "cmp_gt", [c.src(n.args[0])], {"scalar": float(n.args[1])})


@_on("aten.where.self")
def _where(c, n):
    return c.emit(n, "select", [c.src(a) for a in n.args[:3]])


@_on("aten.cat.default")
def _cat(c, n):
    rank = len(_tt(n).shape)
    dim = _dim(int(n.args[1]) if len(n.args) > 1 else 0, rank)
    return c.emit(n, "cat", [c.src(p) for p in n.args[0]], {"dim": dim}, kind="layout")


@_on("aten.constant_pad_nd.default")
def _pad(c, n):
    pads = [int(p) for p in n.args[1]]
    value = float(n.args[2]) if len(n.args) > 2 else 0.0
    return c.emit(n, "pad", [c.src(n.args[0])], {"pad": pads, "value": value})


@_on("aten.convolution.default")
def _conv(c, n):
    x, w, bias, stride, padding, dilation, transposed, out_pad, groups = n.args[:9]
    if transposed or len(_tt(x).shape) != 3:
        raise UnsupportedOpError(f"{n.name}: only non-transposed 1-D convolution")
    ins = [c.src(x), c.src(w)] + ([c.src(bias)] if bias is not None else [])
    return c.emit(n, "conv1d", ins, {"stride": [int(s) for s in stride], "padding": [int(p) for p in padding],
                                     "dilation": [int(d) for d in dilation], "groups": int(groups)})


@_on("aten.embedding.default")
def _embedding(c, n):
    return c.emit(n, "embedding", [c.src(n.args[1]), c.src(n.args[0])])


@_on("aten.linear.default")
def _linear(c, n):
    x, w = n.args[0], n.args[1]
    wt_t = TensorType(tuple(reversed(_tt(w).shape)), _tt(w).dtype)
    wt = c.graph.add("permute", [c.src(w)], wt_t, {"dims": [1, 0]}, kind="layout", name=n.name + "_wT", origin="aten.linear")
    if len(_tt(x).shape) != 2:
        raise UnsupportedOpError(f"{n.name}: linear on a rank-{len(_tt(x).shape)} input")
    if len(n.args) > 2 and n.args[2] is not None:
        mm = c.graph.add("matmul", [c.src(x), wt.name], _tt(n), name=n.name + "_mm", origin="aten.linear")
        return c.emit(n, "add", [mm.name, c.src(n.args[2])])
    return c.emit(n, "matmul", [c.src(x), wt.name])


def fx_to_opgraph(captured: CapturedFx) -> OpGraph:
    return _Converter(captured).run()


def supported_aten_ops() -> list[str]:
    return sorted(_HANDLERS)
