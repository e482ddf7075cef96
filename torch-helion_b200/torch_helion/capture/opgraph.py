"""OpGraph: the single-output operator DAG every compiler stage works on.

The data model and its JSON form are the reference's interchange format
(src/torch_helion/capture/opgraph.py:29-293): ``02_opgraph_raw.json`` and
``03_opgraph_canonical.json`` written here load in the reference and back.
The keys of a node (name, op, kind, inputs, shape, dtype, attrs, origin) and
of a graph (name, inputs, outputs, metadata, nodes) are therefore fixed.

The container itself is this package's: besides the node table it keeps a
consumer index (for every value, how many times each node reads it), so use
counts, consumer lists and use replacement cost O(uses) rather than a sweep
over the graph -- the canonicalisation passes ask those questions for every
candidate match.  Parameter and constant *values* live beside the graph in
``params`` so weight transforms fold at compile time.
"""

from __future__ import annotations

import heapq
import json
import math
from collections import Counter, defaultdict
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Iterable, Iterator

import torch

DTYPE_BYTES = {"float16": 2, "bfloat16": 2, "float32": 4, "float64": 8, "int32": 4, "int64": 8, "bool": 1}
NODE_KINDS = ("input", "param", "const", "compute", "layout")


@dataclass(frozen=True)
class TensorType:
    """Static shape + dtype name (``"float32"``, ``"bfloat16"`` ...)."""

    shape: tuple[int, ...]
    dtype: str = "float16"

    @property
    def rank(self) -> int:
        return len(self.shape)

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n

    @property
    def nbytes(self) -> int:
        return self.numel * DTYPE_BYTES.get(self.dtype, 4)

    @property
    def torch_dtype(self) -> torch.dtype:
        return getattr(torch, self.dtype)

    def with_shape(self, shape: Iterable[int]) -> "TensorType":
        return TensorType(tuple(map(int, shape)), self.dtype)

    @classmethod
    def of(cls, t: torch.Tensor) -> "TensorType":
        return cls(tuple(map(int, t.shape)), str(t.dtype).rsplit(".", 1)[-1])

    def __str__(self) -> str:
        return self.dtype + "[" + ", ".join(map(str, self.shape)) + "]"


@dataclass
class OpNode:
    name: str
    op: str
    inputs: list[str]
    type: TensorType
    attrs: dict[str, Any] = field(default_factory=dict)
    kind: str = "compute"
    origin: str | None = None

    def to_dict(self) -> dict[str, Any]:
        return dict(name=self.name, op=self.op, kind=self.kind, inputs=list(self.inputs),
                    shape=list(self.type.shape), dtype=self.type.dtype, attrs=_to_json_value(self.attrs),
                    origin=self.origin)

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "OpNode":
        return cls(name=d["name"], op=d["op"], inputs=list(d["inputs"]),
                   type=TensorType(tuple(d["shape"]), d["dtype"]), attrs=dict(d.get("attrs") or {}),
                   kind=d.get("kind", "compute"), origin=d.get("origin"))

    def __str__(self) -> str:
        args = ", ".join(self.inputs)
        extra = f" {self.attrs}" if self.attrs else ""
        return f"{self.name}: {self.type} = {self.op}({args}){extra}"


class OpGraph:
    """Nodes in a topological order (insertion order unless re-sorted), the
    graph's input and output value names, parameter values and metadata."""

    def __init__(self, name: str = "graph") -> None:
        self.name = name
        self.nodes: dict[str, OpNode] = {}
        self.inputs: list[str] = []
        self.outputs: list[str] = []
        self.params: dict[str, torch.Tensor] = {}
        self.metadata: dict[str, Any] = {}
        self._readers: dict[str, Counter] = defaultdict(Counter)  # value -> {consumer node: times read}
        self._serial: dict[str, int] = defaultdict(int)          # next suffix per name prefix

    # ------------------------------------------------------------- building
    def fresh_name(self, prefix: str) -> str:
        while True:
            self._serial[prefix] += 1
            cand = f"{prefix}_{self._serial[prefix]}"
            if cand not in self.nodes:
                return cand

    def _index(self, node: OpNode) -> None:
        for i in node.inputs:
            self._readers[i][node.name] += 1

    def _unindex(self, node: OpNode) -> None:
        for i in node.inputs:
            c = self._readers.get(i)
            if c is None:
                continue
            c[node.name] -= 1
            if c[node.name] <= 0:
                del c[node.name]

    def add(self, op: str, inputs: Iterable[str], type: TensorType, attrs: dict | None = None, kind: str = "compute",
            name: str | None = None, origin: str | None = None, value: torch.Tensor | None = None) -> OpNode:
        inputs = list(inputs)
        unknown = [i for i in inputs if i not in self.nodes]
        if unknown:
            raise KeyError(f"{op}: unknown input(s) {unknown}")
        if kind not in NODE_KINDS:
            raise ValueError(f"unknown node kind {kind!r}")
        name = name if name is not None else self.fresh_name(op)
        if name in self.nodes:
            raise KeyError(f"duplicate node name {name!r}")
        node = OpNode(name, op, inputs, type, dict(attrs or {}), kind, origin)
        self.nodes[name] = node
        self._index(node)
        if kind == "input":
            self.inputs.append(name)
        if value is not None:
            self.params[name] = value
        return node

    def add_const(self, value: torch.Tensor, name: str | None = None, origin: str | None = None) -> OpNode:
        return self.add("const", [], TensorType.of(value), kind="const", name=name, origin=origin, value=value)

    # -------------------------------------------------------------- queries
    def __getitem__(self, name: str) -> OpNode:
        return self.nodes[name]

    def __contains__(self, name: str) -> bool:
        return name in self.nodes

    def __iter__(self) -> Iterator[OpNode]:
        return iter(list(self.nodes.values()))

    def __len__(self) -> int:
        return len(self.nodes)

    def users(self, name: str) -> list[OpNode]:
        """Nodes reading ``name`` (each once), in graph order."""
        readers = self._readers.get(name)
        if not readers:
            return []
        return [n for n in self.nodes.values() if n.name in readers]

    def user_map(self) -> dict[str, list[str]]:
        order = {n: k for k, n in enumerate(self.nodes)}
        return {n: sorted(self._readers.get(n, ()), key=order.__getitem__) for n in self.nodes}

    def num_uses(self, name: str) -> int:
        """Reads of ``name`` by nodes (counted per operand slot) plus graph outputs."""
        readers = self._readers.get(name)
        return (sum(readers.values()) if readers else 0) + self.outputs.count(name)

    def value(self, name: str) -> torch.Tensor:
        return self.params[name]

    def is_constant(self, name: str) -> bool:
        return self.nodes[name].kind in ("param", "const")

    # ------------------------------------------------------------- rewriting
    def replace_all_uses(self, old: str, new: str) -> None:
        if old == new:
            return
        for reader in list(self._readers.get(old, ())):
            node = self.nodes[reader]
            self._unindex(node)
            node.inputs = [new if i == old else i for i in node.inputs]
            self._index(node)
        self.outputs = [new if o == old else o for o in self.outputs]

    def redefine(self, name: str, op: str, inputs: Iterable[str], attrs: dict | None = None, kind: str = "compute",
                 type: TensorType | None = None) -> OpNode:
        """Turn node ``name`` into ``op(inputs)`` in place (its readers keep reading it)."""
        node = self.nodes[name]
        self._unindex(node)
        node.op, node.inputs, node.attrs, node.kind = op, list(inputs), dict(attrs or {}), kind
        if type is not None:
            node.type = type
        self._index(node)
        return node

    def _drop(self, name: str) -> None:
        node = self.nodes.pop(name)
        self._unindex(node)
        self._readers.pop(name, None)
        self.params.pop(name, None)
        if name in self.inputs:
            self.inputs.remove(name)

    def remove(self, name: str) -> None:
        if self.num_uses(name):
            raise ValueError(f"cannot remove {name}: still used")
        self._drop(name)

    def dce(self) -> int:
        """Drop every non-input node that no output depends on; returns how
        many.  Reference counting over the consumer index: a node nobody reads
        (and that is not an output) goes, which may leave its operands unread
        in turn.  It does not rely on the node order, which passes may leave
        non-topological until they re-sort."""
        dropped = 0
        work = [n for n, node in self.nodes.items() if node.kind != "input" and self.num_uses(n) == 0]
        while work:
            name = work.pop()
            if name not in self.nodes or self.num_uses(name):
                continue
            operands = set(self.nodes[name].inputs)
            self._drop(name)
            dropped += 1
            work.extend(o for o in operands
                        if o in self.nodes and self.nodes[o].kind != "input" and self.num_uses(o) == 0)
        return dropped

    def toposort(self) -> None:
        """Stable topological order (Kahn): among the nodes whose inputs are
        all placed, the one that came first in the current order goes next."""
        pos = {n: k for k, n in enumerate(self.nodes)}
        pending = {n: len(set(node.inputs)) for n, node in self.nodes.items()}
        ready = [(pos[n], n) for n, k in pending.items() if k == 0]
        heapq.heapify(ready)
        order: list[str] = []
        while ready:
            _, n = heapq.heappop(ready)
            order.append(n)
            for reader in self._readers.get(n, ()):
                pending[reader] -= 1
                if pending[reader] == 0:
                    heapq.heappush(ready, (pos[reader], reader))
        if len(order) != len(self.nodes):
            raise ValueError(f"{self.name}: the graph has a cycle")
        self.nodes = {n: self.nodes[n] for n in order}

    # ---------------------------------------------------------------- output
    def summary(self) -> str:
        head = f"OpGraph {self.name}: {len(self.nodes)} nodes, inputs={self.inputs}, outputs={self.outputs}"
        body = [f"  [{n.kind}] {n.name}: {n.type}" if n.kind in ("param", "const") else f"  {n}"
                for n in self.nodes.values()]
        return "\n".join([head] + body)

    def to_dict(self) -> dict[str, Any]:
        return dict(name=self.name, inputs=list(self.inputs), outputs=list(self.outputs),
                    metadata=_to_json_value(self.metadata), nodes=[n.to_dict() for n in self.nodes.values()])

    def to_json(self, path: str | Path) -> None:
        Path(path).write_text(json.dumps(self.to_dict(), indent=2))

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "OpGraph":
        g = cls(d.get("name", "graph"))
        for nd in d["nodes"]:
            node = OpNode.from_dict(nd)
            g.nodes[node.name] = node
            g._index(node)
        g.inputs = list(d.get("inputs", []))
        g.outputs = list(d.get("outputs", []))
        g.metadata = dict(d.get("metadata", {}))
        return g

    @classmethod
    def from_json(cls, path: str | Path) -> "OpGraph":
        return cls.from_dict(json.loads(Path(path).read_text()))

    def copy(self) -> "OpGraph":
        g = OpGraph.from_dict(self.to_dict())
        g.params = dict(self.params)
        g._serial = defaultdict(int, self._serial)
        return g


def _to_json_value(obj: Any) -> Any:
    """Attribute / metadata values as JSON: torch dtypes by name, non-finite
    floats as strings, anything unknown as its ``str``."""
    if obj is None or isinstance(obj, (bool, int, str)):
        return obj
    if isinstance(obj, float):
        return obj if math.isfinite(obj) else str(obj)
    if isinstance(obj, dict):
        return {str(k): _to_json_value(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return [_to_json_value(v) for v in obj]
    if isinstance(obj, torch.dtype):
        return str(obj).rsplit(".", 1)[-1]
    return str(obj)
