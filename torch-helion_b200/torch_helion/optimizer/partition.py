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

import itertools
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
    """GEMMs reading the same LHS value, one list per LHS, in graph order
    (taken from the graph's consumer index)."""
    sets, done = [], set()
    for node in g:
        if node.op != "matmul" or node.inputs[0] in done:
            continue
        lhs = node.inputs[0]
        done.add(lhs)
        sets.append([u.name for u in g.users(lhs) if u.op == "matmul" and u.inputs[0] == lhs])
    return sets


def default_grouping(g: OpGraph, merge_siblings: bool = True) -> Grouping:
    """Every sibling set in one kernel (or, unmerged, one kernel per GEMM);
    group ids are unique across sets."""
    ids = itertools.count()
    grouping: Grouping = {}
    for members in sibling_sets(g):
        shared = next(ids)
        grouping.update({m: shared if merge_siblings else next(ids) for m in members})
    return grouping


def _ssd_roles(attrs: dict) -> tuple[str, ...]:
    return ("x", "dt", "A", "B", "C") + (("D",) if attrs.get("has_D") else ()) + (("z",) if attrs.get("gate") else ())


@dataclass
class KernelDraft:
    """A kernel while the program is assembled: its spec, the graph values
    computed inside it (value -> the name the kernel body uses for it), where
    it sits in the graph order, and per-kernel caches of bound operands and
    of the row-statistic columns cloned into its epilogue."""

    spec: KernelSpec
    anchor_pos: int
    last_pos: int
    lhs: str | None = None
    local: dict[str, str] = field(default_factory=dict)
    operands: dict[tuple, str] = field(default_factory=dict)
    columns: dict[str, str] = field(default_factory=dict)
    widths: set[int] = field(default_factory=set)

    def computes(self, value: str) -> bool:
        return value in self.local


def _row_stat_source(g: OpGraph, name: str, memo: dict[str, str | None]) -> str | None:
    """``x`` when value ``name`` is built only from ``row_sumsq(x)`` and
    scalars (a per-row column such as an RMSNorm scale), else None."""
    if name not in memo:
        node = g[name]
        found: str | None = None
        if node.op == "row_sumsq":
            found = node.inputs[0]
        elif node.op in BINARY_OPS or node.op in UNARY_OPS:
            sources = {_row_stat_source(g, i, memo) for i in node.inputs}
            if len(sources) == 1 and None not in sources:
                found = next(iter(sources))
        memo[name] = found
    return memo[name]


def _bind(g: OpGraph, name: str) -> tuple[str, list[int] | None]:
    """The tensor and column range a kernel operand reads for value ``name``:
    2-D column slices become a column view of their base tensor."""
    node = g[name]
    if node.kind != "layout":
        return name, None
    if node.op == "slice" and node.attrs.get("dim") == 1 and node.type.rank == 2:
        base, outer = _bind(g, node.inputs[0])
        off = outer[0] if outer else 0
        return base, [off + node.attrs["start"], off + node.attrs["end"]]
    raise PartitionError(f"{name}: layout op {node.op} reaches a kernel boundary")


class _ProgramBuilder:
    """Turns a canonical graph and a grouping into kernels: anchors first
    (GEMM groups, macro ops), then every remaining compute node into the
    epilogue of a GEMM kernel that produces one of its operands, then the
    DRAM outputs, then a dependency order."""

    def __init__(self, g: OpGraph, grouping: Grouping) -> None:
        self.g, self.grouping = g, grouping
        self.pos = {n.name: i for i, n in enumerate(g)}
        self.drafts: dict[tuple, KernelDraft] = {}
        self.home: dict[str, KernelDraft] = {}     # value -> kernel computing it
        self.row_stats: dict[str, str | None] = {}

    # ---- anchors
    def add_gemm(self, n: OpNode) -> None:
        lhs, rhs = n.inputs
        if not _is_const(self.g, rhs):
            raise PartitionError(f"{n.name}: GEMM with a non-constant RHS has no B200 template")
        key = ("gemm", self.grouping[n.name])
        draft = self.drafts.get(key)
        if draft is None:
            spec = KernelSpec(name="", kind="gemm", lhs="lhs", k_extent=self.g[lhs].type.shape[1],
                              grid={"rows": n.type.shape[0], "cols": 0})
            tensor, cols = _bind(self.g, lhs)
            spec.args.append(KernelArg("lhs", tensor, "lhs", cols=cols))
            draft = self.drafts[key] = KernelDraft(spec, self.pos[n.name], self.pos[n.name], lhs=lhs)
        elif draft.lhs != lhs:
            raise PartitionError(f"{n.name}: grouped with GEMMs of a different LHS")
        spec = draft.spec
        weight = f"w{len(spec.gemms)}"
        spec.args.append(KernelArg(weight, rhs, "rhs"))
        spec.gemms.append(GemmSpec(f"acc_{n.name}", weight))
        spec.grid["cols"] += n.type.shape[1]
        draft.widths.add(n.type.shape[1])
        draft.local[n.name] = f"acc_{n.name}"
        self.home[n.name] = draft

    def add_macro(self, n: OpNode) -> None:
        roles = _ssd_roles(n.attrs) if n.op == "ssd" else MACRO_ANCHORS[n.op]
        if len(roles) != len(n.inputs):
            raise PartitionError(f"{n.name}: {n.op} expects inputs {roles}")
        spec = KernelSpec(name="", kind=n.op, attrs=dict(n.attrs))
        for role, value in zip(roles, n.inputs):
            tensor, cols = _bind(self.g, value)
            spec.args.append(KernelArg(role, tensor, role, cols=cols))
        draft = self.drafts[("macro", n.name)] = KernelDraft(spec, self.pos[n.name], self.pos[n.name])
        draft.local[n.name] = "out"
        self.home[n.name] = draft

    # ---- epilogues
    def is_row_column(self, name: str) -> bool:
        node = self.g[name]
        if _row_stat_source(self.g, name, self.row_stats) is not None:
            return True
        return node.op == "broadcast" and _row_stat_source(self.g, node.inputs[0], self.row_stats) is not None

    def place(self, n: OpNode) -> None:
        fits = [self.home[i] for i in n.inputs
                if i in self.home and self.home[i].spec.kind == "gemm"
                and n.type.shape[0] == self.home[i].spec.grid["rows"] and n.type.shape[1] in self.home[i].widths]
        if not fits:
            raise PartitionError(f"{n.name} ({n.op}): elementwise op with no GEMM epilogue to live in")
        draft = max(fits, key=lambda d: d.anchor_pos)  # the latest-anchored producer
        draft.last_pos = max(draft.last_pos, self.pos[n.name])
        operands = [self.operand(draft, i) for i in n.inputs]
        draft.spec.epilogue.append(BodyOp(n.name, n.op, operands, dict(n.attrs)))
        draft.local[n.name] = n.name
        self.home[n.name] = draft

    def operand(self, draft: KernelDraft, value: str) -> str:
        """The epilogue name of ``value`` inside ``draft``: computed there, a
        row column rebuilt from the kernel's own Σx², or a bound input."""
        if value in draft.local:
            return draft.local[value]
        if _row_stat_source(self.g, value, self.row_stats) is not None:
            return self.column(draft, value)
        node = self.g[value]
        if node.op == "broadcast" and _row_stat_source(self.g, node.inputs[0], self.row_stats) is not None:
            inner = self.column(draft, node.inputs[0])
            key = f"bcast:{inner}:{node.attrs.get('shape')}"
            if key not in draft.columns:
                local = f"{node.name}__{len(draft.columns)}"
                draft.spec.epilogue.append(BodyOp(local, "broadcast", [inner], dict(node.attrs)))
                draft.columns[key] = local
            draft.local[value] = draft.columns[key]
            return draft.local[value]
        tensor, cols = _bind(self.g, value)
        key = (tensor, tuple(cols) if cols else None)
        if key not in draft.operands:
            name = f"in{len(draft.operands)}"
            draft.spec.args.append(KernelArg(name, tensor, "const" if _is_const(self.g, tensor) else "extra", cols=cols))
            draft.operands[key] = name
        return draft.operands[key]

    def column(self, draft: KernelDraft, value: str) -> str:
        """Rebuild a row-statistic column inside ``draft`` from its LHS Σx²."""
        if value in draft.columns:
            return draft.columns[value]
        node = self.g[value]
        if node.op == "row_sumsq":
            if draft.lhs != node.inputs[0]:
                raise PartitionError(f"needs the row sum of squares of {node.inputs[0]} but the kernel's LHS "
                                     f"is {draft.lhs}")
            draft.spec.sumsq = True
            draft.columns[value] = "sumsq"
        else:
            operands = [self.column(draft, i) for i in node.inputs]
            local = f"{value}__col"
            draft.spec.epilogue.append(BodyOp(local, node.op, operands, dict(node.attrs)))
            draft.columns[value] = local
        return draft.columns[value]

    # ---- outputs and order
    def assign_outputs(self) -> None:
        readers: dict[str, set[int]] = {}
        for d in self.drafts.values():
            for a in d.spec.args:
                readers.setdefault(a.tensor, set()).add(id(d))
        for value, d in list(self.home.items()):
            if d.spec.kind != "gemm":
                d.spec.outputs = [KernelOutput(value, "out")]
                continue
            leaves = value in self.g.outputs
            leaves = leaves or any(u.name not in d.local for u in self.g.users(value) if u.kind in ("compute", "layout"))
            leaves = leaves or any(r != id(d) for r in readers.get(value, ()))
            if leaves and d.local[value] and value not in d.spec.output_tensors():
                d.spec.outputs.append(KernelOutput(value, d.local[value]))

    def ordered(self) -> list[KernelDraft]:
        """Kernels in dependency order, ties broken by graph position."""
        producer = {o.tensor: d for d in self.drafts.values() for o in d.spec.outputs}
        pending = sorted(self.drafts.values(), key=lambda d: d.last_pos)
        placed: list[KernelDraft] = []
        placed_ids: set[int] = set()
        while pending:
            ready = next((d for d in pending
                          if all(id(producer[a.tensor]) in placed_ids
                                 for a in d.spec.args if a.tensor in producer and producer[a.tensor] is not d)), None)
            if ready is None:
                raise PartitionError("cyclic kernel dependencies")
            pending.remove(ready)
            placed.append(ready)
            placed_ids.add(id(ready))
        return placed


def build_program(g: OpGraph, grouping: Grouping | None = None, name: str = "program") -> Program:
    b = _ProgramBuilder(g, grouping if grouping is not None else default_grouping(g))
    for n in g:
        if n.op == "matmul":
            b.add_gemm(n)
        elif n.op in MACRO_ANCHORS or n.op == "ssd":
            b.add_macro(n)
        elif n.op == "batch_matmul":
            raise PartitionError(f"{n.name}: standalone batch_matmul has no B200 template")
    for n in g:
        if n.kind == "compute" and n.name not in b.home and n.op != "row_sumsq" and not b.is_row_column(n.name):
            b.place(n)
    b.assign_outputs()
    drafts = b.ordered()
    for i, d in enumerate(drafts):
        d.spec.name = f"k{i}_{d.spec.kind}"
    params = sorted({a.tensor for d in drafts for a in d.spec.args if _is_const(g, a.tensor)})
    prog = Program(name=name, inputs=list(g.inputs), outputs=list(g.outputs), tensors={n.name: n.type for n in g},
                   kernels=[d.spec for d in drafts], params=params, metadata=dict(g.metadata))
    prog.metadata["grouping"] = dict(b.grouping)
    return prog
