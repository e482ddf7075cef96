"""Partition the canonical OpGraph into B200 kernels (an OpIR Program).

Anchors, as in the reference partitioner (src/torch_helion/optimizer/
partition.py:99-229): a group of GEMMs sharing their LHS becomes one
``gemm`` kernel; every macro op (``attention``, ``ssd``,
``causal_conv1d``, ``rmsnorm``, ``embedding``) anchors its own kernel.
Elementwise ops, broadcasts and the RMSNorm row-scale column are pulled
into the epilogue of the GEMM kernel that produces their operands, and a
value crossing kernels becomes a DRAM tensor.  Differences for B200:

* sibling GEMMs need not share their output width -- they are
  concatenated along N into one wide GEMM whose epilogue works per column
  segment;
* a ``slice`` of a token-major tensor is bound as a column view
  (``KernelArg.cols``) instead of being rejected.

Which siblings share a kernel (the *grouping*) is the planner's choice;
:func:`build_program` is deterministic given a grouping.
"""

from __future__ import annotations

from dataclasses import dataclass, field

from ..capture.opgraph import OpGraph, OpNode, TensorType
from ..capture.ops import BINARY_OPS, UNARY_OPS
from .opir import BodyOp, GemmSpec, KernelArg, KernelOutput, KernelSpec, Program


class PartitionError(RuntimeError):
    pass


Grouping = dict[str, int]

MACRO_ANCHORS = {
    "attention": ("q", "k", "v"),
    "causal_conv1d": ("x", "w"),
    "rmsnorm": ("x", "gain"),
    "embedding": ("ids", "table"),
}


def _is_const(g: OpGraph, name: str) -> bool:
    return g[name].kind in ("param", "const")


def sibling_sets(g: OpGraph) -> list[list[str]]:
    """GEMMs sharing the same LHS tensor, in graph order."""
    by_lhs: dict[str, list[str]] = {}
    for n in g:
        if n.op == "matmul":
            by_lhs.setdefault(n.inputs[0], []).append(n.name)
    return list(by_lhs.values())


def default_grouping(g: OpGraph, merge_siblings: bool = True) -> Grouping:
    grouping: Grouping = {}
    gid = 0
    for group in sibling_sets(g):
        for m in group:
            grouping[m] = gid
            if not merge_siblings:
                gid += 1
        if merge_siblings:
            gid += 1
    return grouping


def _ssd_roles(attrs: dict) -> tuple[str, ...]:
    roles = ["x", "dt", "A", "B", "C"]
    if attrs.get("has_D"):
        roles.append("D")
    if attrs.get("gate"):
        roles.append("z")
    return tuple(roles)


@dataclass
class _K:
    spec: KernelSpec
    owned: dict[str, str] = field(default_factory=dict)
    order_key: int = 0
    anchor_key: int = 0
    lhs_node: str | None = None
    extra: dict[str, str] = field(default_factory=dict)
    column_cache: dict[str, str] = field(default_factory=dict)
    widths: set[int] = field(default_factory=set)


def _is_column_chain(g: OpGraph, name: str, memo: dict[str, str | None]) -> str | None:
    """``x`` when ``name`` derives only from ``row_sumsq(x)`` and scalars."""
    if name in memo:
        return memo[name]
    node = g[name]
    res: str | None = None
    if node.op == "row_sumsq":
        res = node.inputs[0]
    elif node.op in BINARY_OPS or node.op in UNARY_OPS:
        srcs = {_is_column_chain(g, i, memo) for i in node.inputs}
        if None not in srcs and len(srcs) == 1:
            res = srcs.pop()
    memo[name] = res
    return res


def _bind(g: OpGraph, name: str) -> tuple[str, list[int] | None]:
    """Tensor + column range a kernel argument reads for graph value ``name``."""
    node = g[name]
    if node.kind == "layout" and node.op == "slice" and node.attrs.get("dim") == 1 and node.type.rank == 2:
        base, cols = _bind(g, node.inputs[0])
        lo, hi = node.attrs["start"], node.attrs["end"]
        if cols:
            lo, hi = cols[0] + lo, cols[0] + hi
        return base, [lo, hi]
    if node.kind == "layout":
        raise PartitionError(f"{name}: layout op {node.op} reaches a kernel boundary")
    return name, None


def build_program(g: OpGraph, grouping: Grouping | None = None, name: str = "program") -> Program:
    grouping = grouping if grouping is not None else default_grouping(g)
    order = {n.name: i for i, n in enumerate(g)}
    kernels: dict[object, _K] = {}
    owner: dict[str, _K] = {}
    memo: dict[str, str | None] = {}
    tensors: dict[str, TensorType] = {n.name: n.type for n in g}

    # ---- anchors
    for n in g:
        if n.op == "matmul":
            lhs, rhs = n.inputs
            if not _is_const(g, rhs):
                raise PartitionError(f"{n.name}: GEMM with a non-constant RHS has no B200 template")
            key = ("gemm", grouping[n.name])
            if key not in kernels:
                spec = KernelSpec(name="", kind="gemm", lhs="lhs", k_extent=g[lhs].type.shape[1],
                                  grid={"rows": n.type.shape[0], "cols": 0})
                lt, lcols = _bind(g, lhs)
                spec.args.append(KernelArg("lhs", lt, "lhs", cols=lcols))
                kernels[key] = _K(spec, lhs_node=lhs, order_key=order[n.name], anchor_key=order[n.name])
            k = kernels[key]
            if k.lhs_node != lhs:
                raise PartitionError(f"{n.name}: grouped with GEMMs of a different LHS")
            arg = f"w{len(k.spec.gemms)}"
            k.spec.args.append(KernelArg(arg, rhs, "rhs"))
            acc = f"acc_{n.name}"
            k.spec.gemms.append(GemmSpec(acc, arg))
            k.spec.grid["cols"] += n.type.shape[1]
            k.widths.add(n.type.shape[1])
            k.owned[n.name] = acc
            owner[n.name] = k
        elif n.op in MACRO_ANCHORS or n.op == "ssd":
            roles = _ssd_roles(n.attrs) if n.op == "ssd" else MACRO_ANCHORS[n.op]
            if len(roles) != len(n.inputs):
                raise PartitionError(f"{n.name}: {n.op} expects inputs {roles}")
            spec = KernelSpec(name="", kind=n.op, attrs=dict(n.attrs))
            for role, src in zip(roles, n.inputs):
                t, cols = _bind(g, src)
                spec.args.append(KernelArg(role, t, role, cols=cols))
            k = _K(spec, order_key=order[n.name], anchor_key=order[n.name])
            k.owned[n.name] = "out"
            kernels[("macro", n.name)] = k
            owner[n.name] = k
        elif n.op == "batch_matmul":
            raise PartitionError(f"{n.name}: standalone batch_matmul has no B200 template")

    # ---- epilogue placement
    for n in g:
        if n.kind != "compute" or n.op in ("matmul", "row_sumsq") or n.op in MACRO_ANCHORS or n.op == "ssd":
            continue
        if _is_column_chain(g, n.name, memo) is not None:
            continue
        if n.op == "broadcast" and _is_column_chain(g, n.inputs[0], memo) is not None:
            continue  # a row-scale broadcast is cloned into each consumer on demand
        homes = [owner[i] for i in n.inputs if i in owner and owner[i].spec.kind == "gemm"
                 and n.type.shape[0] == owner[i].spec.grid["rows"] and n.type.shape[1] in owner[i].widths]
        if not homes:
            raise PartitionError(f"{n.name} ({n.op}): elementwise op with no GEMM epilogue to live in")
        home = max(homes, key=lambda k: k.anchor_key)
        home.order_key = max(home.order_key, order[n.name])
        ins = [_materialize(g, i, home, memo) for i in n.inputs]
        home.spec.epilogue.append(BodyOp(n.name, n.op, ins, dict(n.attrs)))
        home.owned[n.name] = n.name
        owner[n.name] = home

    # ---- outputs
    consumers: dict[str, set[int]] = {}
    for k in kernels.values():
        for a in k.spec.args:
            consumers.setdefault(a.tensor, set()).add(id(k))
    for value, k in list(owner.items()):
        if k.spec.kind != "gemm":
            k.spec.outputs = [KernelOutput(value, "out")]
            continue
        used_outside = value in g.outputs or any(
            u.name not in k.owned for u in g.users(value) if u.kind == "compute" or u.kind == "layout")
        used_outside = used_outside or any(c != id(k) for c in consumers.get(value, ()))
        if used_outside and k.owned[value] and value not in k.spec.output_tensors():
            k.spec.outputs.append(KernelOutput(value, k.owned[value]))

    ordered = _order_kernels(list(kernels.values()))
    for i, k in enumerate(ordered):
        k.spec.name = f"k{i}_{k.spec.kind}"
    params = sorted({a.tensor for k in ordered for a in k.spec.args if _is_const(g, a.tensor)})
    prog = Program(name=name, inputs=list(g.inputs), outputs=list(g.outputs), tensors=tensors,
                   kernels=[k.spec for k in ordered], params=params, metadata=dict(g.metadata))
    prog.metadata["grouping"] = dict(grouping)
    return prog


def _materialize(g: OpGraph, src: str, home: _K, memo: dict) -> str:
    if src in home.owned:
        return home.owned[src]
    if _is_column_chain(g, src, memo) is not None:
        return _clone_column(g, src, home, memo)
    node = g[src]
    if node.op == "broadcast" and _is_column_chain(g, node.inputs[0], memo) is not None:
        inner = _clone_column(g, node.inputs[0], home, memo)
        key = f"bcast:{inner}:{node.attrs.get('shape')}"
        if key not in home.column_cache:
            bn = f"{node.name}__{len(home.column_cache)}"
            home.spec.epilogue.append(BodyOp(bn, "broadcast", [inner], dict(node.attrs)))
            home.column_cache[key] = bn
        home.owned[src] = home.column_cache[key]
        return home.column_cache[key]
    t, cols = _bind(g, src)
    key = f"{t}:{cols}"
    if key in home.extra:
        return home.extra[key]
    arg = f"in{len(home.extra)}"
    role = "const" if _is_const(g, t) else "extra"
    home.spec.args.append(KernelArg(arg, t, role, cols=cols))
    home.extra[key] = arg
    return arg


def _clone_column(g: OpGraph, name: str, home: _K, memo: dict) -> str:
    if name in home.column_cache:
        return home.column_cache[name]
    node = g[name]
    if node.op == "row_sumsq":
        if home.lhs_node != node.inputs[0]:
            raise PartitionError(f"needs the row sum of squares of {node.inputs[0]} but the kernel's LHS is {home.lhs_node}")
        home.spec.sumsq = True
        home.column_cache[name] = "sumsq"
        return "sumsq"
    ins = [_clone_column(g, i, home, memo) for i in node.inputs]
    local = f"{name}__col"
    home.spec.epilogue.append(BodyOp(local, node.op, ins, dict(node.attrs)))
    home.column_cache[name] = local
    return local


def _order_kernels(kernels: list[_K]) -> list[_K]:
    produced = {o.tensor: k for k in kernels for o in k.spec.outputs}
    done: list[_K] = []
    remaining = sorted(kernels, key=lambda k: k.order_key)
    while remaining:
        progressed = False
        for k in list(remaining):
            deps = [produced[a.tensor] for a in k.spec.args if a.tensor in produced and produced[a.tensor] is not k]
            if all(d in done for d in deps):
                done.append(k)
                remaining.remove(k)
                progressed = True
        if not progressed:
            raise PartitionError("cyclic kernel dependencies")
    return done
