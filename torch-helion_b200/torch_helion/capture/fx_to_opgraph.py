"""Core-ATen FX graph -> raw OpGraph.

The raw graph is a literal image of the exported program, as the reference
specifies it (src/torch_helion/capture/fx_to_opgraph.py:80-121): one OpGraph
node per ATen call with the call's static shape, layout calls kept as
``layout`` nodes, parameters / buffers / lifted constants as value nodes
carrying their tensors, and every semantic rewrite left to the optimizer.
Anything without a mapping raises :class:`UnsupportedOpError` (the
reference's behaviour for unknown ops, fx_to_opgraph.py:107-109).

How it is organised here: the graph signature's input specs bind the
placeholders; every ``call_function`` is looked up by its overload name
("add.Tensor", "mean.dim", ...) in one of three tables -- elementwise ops
(unary, or binary with an optional scalar operand), ops whose attributes are
read by a small decoder, and expansions that emit more than one node
(``addmm``, ``linear``) or none (``split_with_sizes``, resolved when its
``getitem`` users are met).  Beyond the reference's op set it maps
``constant_pad_nd``, ``convolution`` (Mamba's depthwise causal conv),
``embedding``, ``erf`` and ``gelu``.
"""

from __future__ import annotations

from typing import Any, Callable

import torch
from torch.export.graph_signature import InputKind
from torch.fx import Node

from .fx_capture import CapturedFx
from .opgraph import OpGraph, OpNode, TensorType


class UnsupportedOpError(NotImplementedError):
    """An ATen op has no OpGraph mapping."""


def _overload(target: Any) -> str:
    """'aten.add.Tensor' -> 'add.Tensor'; the getitem builtin -> 'getitem'."""
    text = str(target)
    if text.startswith("aten."):
        return text[len("aten."):]
    return "getitem" if "getitem" in text else text


def _type_of(node: Node) -> TensorType:
    val = node.meta.get("val")
    if not isinstance(val, torch.Tensor):
        raise UnsupportedOpError(f"{node.name}: produces {type(val).__name__}, not a tensor")
    return TensorType.of(val)


def _axis(node: Node, axis: int) -> int:
    """A possibly negative axis of ``node``'s value, made non-negative."""
    rank = len(_type_of(node).shape)
    return axis % rank if rank else 0


def _arg(node: Node, pos: int, key: str, default: Any) -> Any:
    if len(node.args) > pos and node.args[pos] is not None:
        return node.args[pos]
    return node.kwargs.get(key, default)


# Elementwise ops: one OpGraph op per overload.
_UNARY = {
    "exp.default": "exp", "log.default": "log", "neg.default": "neg", "rsqrt.default": "rsqrt",
    "sqrt.default": "sqrt", "sigmoid.default": "sigmoid", "silu.default": "silu", "tanh.default": "tanh",
    "square.default": "square", "log1p.default": "log1p", "erf.default": "erf",
}
_BINARY = {
    "add.Tensor": "add", "sub.Tensor": "sub", "mul.Tensor": "mul", "div.Tensor": "div", "maximum.default": "max",
    "pow.Tensor_Tensor": "powf",
}
_REDUCTIONS = {"mean.dim": "row_mean", "sum.dim_IntList": "row_sum", "amax.default": "row_max"}
_VIEWS = ("view.default", "reshape.default", "_unsafe_view.default", "unsqueeze.default", "squeeze.dim",
          "squeeze.default", "squeeze.dims")
_COPIES = ("clone.default", "contiguous.default", "alias.default", "detach.default")


class _Lowering:
    def __init__(self, captured: CapturedFx) -> None:
        self.captured = captured
        self.program = captured.exported
        self.graph = OpGraph("model")
        self.value_of: dict[str, str] = {}                       # fx node -> OpGraph value
        self.pending_splits: dict[str, tuple[str, list[int], int]] = {}

    # ---------------------------------------------------------------- helpers
    def operand(self, arg: Any) -> str:
        if not isinstance(arg, Node):
            raise UnsupportedOpError(f"expected a tensor operand, got {arg!r}")
        return self.value_of[arg.name]

    def node(self, fx: Node, op: str, inputs: list[str], attrs: dict | None = None, kind: str = "compute") -> OpNode:
        out = self.graph.add(op, inputs, _type_of(fx), attrs=attrs, kind=kind, name=fx.name, origin=str(fx.target))
        self.value_of[fx.name] = out.name
        return out

    def helper(self, fx: Node, suffix: str, op: str, inputs: list[str], t: TensorType, attrs: dict | None = None,
               kind: str = "compute") -> OpNode:
        """An extra node of a multi-node expansion (named after the FX node)."""
        return self.graph.add(op, inputs, t, attrs=attrs, kind=kind, name=f"{fx.name}_{suffix}",
                              origin=f"aten.{_overload(fx.target).split('.')[0]}")

    # ------------------------------------------------------------- placeholders
    def bind_inputs(self) -> None:
        ep = self.program
        state, consts = dict(ep.state_dict), dict(getattr(ep, "constants", {}) or {})
        placeholders = {n.name: n for n in ep.graph_module.graph.nodes if n.op == "placeholder"}
        for spec in ep.graph_signature.input_specs:
            fx = placeholders[spec.arg.name]
            t = _type_of(fx)
            if spec.kind == InputKind.USER_INPUT:
                kind, label, value = "input", fx.name, None
            elif spec.kind in (InputKind.PARAMETER, InputKind.BUFFER):
                kind, label = "param", spec.target
                value = state[label] if label in state else consts.get(label)
            elif spec.kind == InputKind.CONSTANT_TENSOR:
                kind, label, value = "const", spec.target, consts[spec.target]
            else:
                raise UnsupportedOpError(f"placeholder {fx.name}: input kind {spec.kind} is not supported")
            stored = None if value is None else value.detach().clone()
            out = self.graph.add(kind, [], t, kind=kind, name=label.replace(".", "_"), origin=fx.name, value=stored)
            self.value_of[fx.name] = out.name

    # ------------------------------------------------------------------ calls
    def lower(self, fx: Node) -> None:
        key = _overload(fx.target)
        if key in _UNARY:
            self.node(fx, _UNARY[key], [self.operand(fx.args[0])])
        elif key in _BINARY:
            self.binary(fx, _BINARY[key])
        elif key in _REDUCTIONS:
            self.reduction(fx, _REDUCTIONS[key])
        elif key in _VIEWS:
            self.node(fx, "view", [self.operand(fx.args[0])], {"shape": list(_type_of(fx).shape)}, kind="layout")
        elif key in _COPIES:
            self.node(fx, "clone", [self.operand(fx.args[0])], kind="layout")
        elif key in _DECODERS:
            op, kind, decode = _DECODERS[key]
            inputs, attrs = decode(self, fx)
            self.node(fx, op, inputs, attrs, kind=kind)
        elif key in _EXPANSIONS:
            _EXPANSIONS[key](self, fx)
        else:
            raise UnsupportedOpError(f"no OpGraph mapping for aten.{key} (node {fx.name})")

    def binary(self, fx: Node, op: str) -> None:
        lhs, rhs = fx.args[0], fx.args[1]
        tensors = [a for a in (lhs, rhs) if isinstance(a, Node)]
        if len(tensors) == 2:
            self.node(fx, op, [self.operand(lhs), self.operand(rhs)])
        elif isinstance(lhs, Node):
            self.node(fx, op, [self.operand(lhs)], {"scalar": float(rhs)})
        else:  # scalar (op) tensor: the order matters for sub/div/pow
            self.node(fx, op, [self.operand(rhs)], {"scalar": float(lhs), "scalar_first": True})

    def reduction(self, fx: Node, op: str) -> None:
        src = fx.args[0]
        rank = len(_type_of(src).shape)
        raw = _arg(fx, 1, "dim", None)
        axes = sorted({(int(d) % rank) for d in ([raw] if isinstance(raw, int) else (raw or []))})
        if axes != [rank - 1]:
            raise UnsupportedOpError(f"{fx.name}: only last-axis reductions are supported (axes {axes})")
        self.node(fx, op, [self.operand(src)], {"keepdim": bool(_arg(fx, 2, "keepdim", False))})

    # ------------------------------------------------------------------ driver
    def run(self) -> OpGraph:
        self.bind_inputs()
        for fx in self.program.graph_module.graph.nodes:
            if fx.op == "placeholder":
                continue
            if fx.op == "call_function":
                if _overload(fx.target) == "split_with_sizes.default":
                    src = fx.args[0]
                    axis = _axis(src, int(_arg(fx, 2, "dim", 0)))
                    self.pending_splits[fx.name] = (self.operand(src), [int(v) for v in fx.args[1]], axis)
                else:
                    self.lower(fx)
            elif fx.op == "output":
                results = fx.args[0] if isinstance(fx.args[0], (tuple, list)) else (fx.args[0],)
                self.graph.outputs = [self.operand(r) for r in results]
            else:
                raise UnsupportedOpError(f"unsupported fx node kind {fx.op} ({fx.target})")
        self.graph.metadata["fx_op_histogram"] = self.captured.op_histogram()
        return self.graph


# ------------------------------------------------- decoders: (inputs, attrs)
def _dec_pow_scalar(lw: _Lowering, fx: Node):
    return [lw.operand(fx.args[0])], {"scalar": float(fx.args[1])}


def _dec_softmax(lw: _Lowering, fx: Node):
    if _axis(fx.args[0], int(fx.args[1])) != len(_type_of(fx.args[0]).shape) - 1:
        raise UnsupportedOpError(f"{fx.name}: softmax only over the last axis")
    return [lw.operand(fx.args[0])], {}


def _dec_two(lw: _Lowering, fx: Node):
    return [lw.operand(fx.args[0]), lw.operand(fx.args[1])], {}


def _dec_permute(lw: _Lowering, fx: Node):
    return [lw.operand(fx.args[0])], {"dims": [int(d) for d in fx.args[1]]}


def _dec_transpose(lw: _Lowering, fx: Node):
    src = fx.args[0]
    order = list(range(len(_type_of(src).shape)))
    a, b = _axis(src, int(fx.args[1])), _axis(src, int(fx.args[2]))
    order[a], order[b] = order[b], order[a]
    return [lw.operand(src)], {"dims": order}


def _dec_t(lw: _Lowering, fx: Node):
    return [lw.operand(fx.args[0])], {"dims": [1, 0]}


def _dec_expand(lw: _Lowering, fx: Node):
    return [lw.operand(fx.args[0])], {"shape": list(_type_of(fx).shape)}


def _dec_cast(lw: _Lowering, fx: Node):
    return [lw.operand(fx.args[0])], {"dtype": _type_of(fx).dtype}


def _dec_slice(lw: _Lowering, fx: Node):
    src = fx.args[0]
    axis = _axis(src, int(_arg(fx, 1, "dim", 0)))
    extent = _type_of(src).shape[axis]
    if int(_arg(fx, 4, "step", 1)) != 1:
        raise UnsupportedOpError(f"{fx.name}: strided slice")
    lo, hi = int(_arg(fx, 2, "start", 0)), int(_arg(fx, 3, "end", extent))
    lo, hi = (lo + extent if lo < 0 else lo), (hi + extent if hi < 0 else hi)
    return [lw.operand(src)], {"dim": axis, "start": max(0, lo), "end": min(extent, hi)}


def _dec_getitem(lw: _Lowering, fx: Node):
    parent, index = fx.args[0], int(fx.args[1])
    if not isinstance(parent, Node) or parent.name not in lw.pending_splits:
        raise UnsupportedOpError(f"{fx.name}: getitem on something other than a tensor split")
    base, sizes, axis = lw.pending_splits[parent.name]
    lo = sum(sizes[:index])
    return [base], {"dim": axis, "start": lo, "end": lo + sizes[index]}


def _dec_cumsum(lw: _Lowering, fx: Node):
    src = fx.args[0]
    if _axis(src, int(_arg(fx, 1, "dim", -1))) != len(_type_of(src).shape) - 1:
        raise UnsupportedOpError(f"{fx.name}: only last-axis cumsum")
    return [lw.operand(src)], {}


def _dec_gt(lw: _Lowering, fx: Node):
    return [lw.operand(fx.args[0])], {"scalar": float(fx.args[1])}


def _dec_where(lw: _Lowering, fx: Node):
    return [lw.operand(a) for a in fx.args[:3]], {}


def _dec_cat(lw: _Lowering, fx: Node):
    return [lw.operand(p) for p in fx.args[0]], {"dim": _axis(fx, int(_arg(fx, 1, "dim", 0)))}


def _dec_pad(lw: _Lowering, fx: Node):
    return [lw.operand(fx.args[0])], {"pad": [int(p) for p in fx.args[1]], "value": float(_arg(fx, 2, "value", 0.0))}


def _dec_conv(lw: _Lowering, fx: Node):
    x, w, bias, stride, padding, dilation, transposed, _out_pad, groups = fx.args[:9]
    if transposed or len(_type_of(x).shape) != 3:
        raise UnsupportedOpError(f"{fx.name}: only non-transposed 1-D convolution")
    inputs = [lw.operand(x), lw.operand(w)] + ([lw.operand(bias)] if bias is not None else [])
    return inputs, {"stride": list(map(int, stride)), "padding": list(map(int, padding)),
                    "dilation": list(map(int, dilation)), "groups": int(groups)}


def _dec_embedding(lw: _Lowering, fx: Node):
    table, ids = fx.args[0], fx.args[1]
    return [lw.operand(ids), lw.operand(table)], {}


def _dec_gelu(lw: _Lowering, fx: Node):
    approx = str(_arg(fx, 1, "approximate", "none"))
    if approx not in ("none", "tanh"):
        raise UnsupportedOpError(f"{fx.name}: gelu approximate={approx!r}")
    return [lw.operand(fx.args[0])], {"approximate": approx}


# overload -> (OpGraph op, node kind, decoder)
_DECODERS: dict[str, tuple[str, str, Callable[[_Lowering, Node], tuple[list[str], dict]]]] = {
    "pow.Tensor_Scalar": ("powf", "compute", _dec_pow_scalar),
    "_softmax.default": ("softmax", "compute", _dec_softmax),
    "softmax.int": ("softmax", "compute", _dec_softmax),
    "mm.default": ("matmul", "compute", _dec_two),
    "bmm.default": ("batch_matmul", "compute", _dec_two),
    "permute.default": ("permute", "layout", _dec_permute),
    "transpose.int": ("permute", "layout", _dec_transpose),
    "t.default": ("permute", "layout", _dec_t),
    "expand.default": ("expand", "layout", _dec_expand),
    "_to_copy.default": ("cast", "layout", _dec_cast),
    "to.dtype": ("cast", "layout", _dec_cast),
    "slice.Tensor": ("slice", "layout", _dec_slice),
    "getitem": ("slice", "layout", _dec_getitem),
    "cumsum.default": ("row_cumsum", "compute", _dec_cumsum),
    "gt.Scalar": ("cmp_gt", "compute", _dec_gt),
    "where.self": ("select", "compute", _dec_where),
    "cat.default": ("cat", "layout", _dec_cat),
    "constant_pad_nd.default": ("pad", "compute", _dec_pad),
    "convolution.default": ("conv1d", "compute", _dec_conv),
    "embedding.default": ("embedding", "compute", _dec_embedding),
    "gelu.default": ("gelu", "compute", _dec_gelu),
}


# ------------------------------------------- expansions (several nodes each)
def _exp_addmm(lw: _Lowering, fx: Node) -> None:
    bias, a, b = fx.args[:3]
    prod = lw.helper(fx, "mm", "matmul", [lw.operand(a), lw.operand(b)], _type_of(fx))
    lw.node(fx, "add", [prod.name, lw.operand(bias)])


def _exp_linear(lw: _Lowering, fx: Node) -> None:
    x, w = fx.args[0], fx.args[1]
    bias = _arg(fx, 2, "bias", None)
    if len(_type_of(x).shape) != 2:
        raise UnsupportedOpError(f"{fx.name}: linear on a rank-{len(_type_of(x).shape)} input")
    wt = _type_of(w)
    w_t = lw.helper(fx, "wT", "permute", [lw.operand(w)], TensorType(wt.shape[::-1], wt.dtype), {"dims": [1, 0]},
                    kind="layout")
    if bias is None:
        lw.node(fx, "matmul", [lw.operand(x), w_t.name])
        return
    prod = lw.helper(fx, "mm", "matmul", [lw.operand(x), w_t.name], _type_of(fx))
    lw.node(fx, "add", [prod.name, lw.operand(bias)])


_EXPANSIONS: dict[str, Callable[[_Lowering, Node], None]] = {
    "addmm.default": _exp_addmm,
    "linear.default": _exp_linear,
}


def fx_to_opgraph(captured: CapturedFx) -> OpGraph:
    return _Lowering(captured).run()


def supported_aten_ops() -> list[str]:
    keys = list(_UNARY) + list(_BINARY) + list(_REDUCTIONS) + list(_VIEWS) + list(_COPIES) + list(_DECODERS) \
        + list(_EXPANSIONS) + ["split_with_sizes.default"]
    return sorted(k if k == "getitem" else f"aten.{k}" for k in keys)
