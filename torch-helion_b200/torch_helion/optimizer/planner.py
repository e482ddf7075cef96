"""Planner: choose which sibling GEMMs share a kernel, by the B200 cost model.

What the search covers is the reference planner's contract
(src/torch_helion/optimizer/planner.py:70-164): for every set of sibling
GEMMs (same LHS) any way of splitting the set into kernels is a candidate,
each candidate program is checked for legality and costed kernel by kernel
plus a launch overhead per kernel, and the cheapest legal program wins.
``planner_mode="greedy"`` only tries all-merged and all-split per set.

How it is searched here:

* a split of a sibling set is a *restricted growth string* (RGS): member i
  gets block label ``a[i] <= 1 + max(a[:i])``; the RGS of length n
  enumerate the Bell(n) set partitions exactly once, iteratively;
* a candidate is one RGS per sibling set; small products are searched
  exhaustively, large ones (deep models: one set per projection per layer)
  by coordinate descent from all-merged -- a set's split changes only its
  own kernels and the cost is a sum over kernels, so the descent converges
  to the same optimum;
* kernel costs are memoised on a structural key (kind, attributes, operand
  shapes and roles, epilogue), so equal layers are costed once.
"""

from __future__ import annotations

import hashlib
import itertools
from dataclasses import dataclass, field
from typing import Any, Iterator, Sequence

from ..capture.opgraph import OpGraph
from ..cost_models.b200 import B200Spec, CostModelError, search_tiles
from .legality import check_program
from .opir import Program
from .partition import Grouping, PartitionError, build_program, sibling_sets


@dataclass
class Candidate:
    index: int
    grouping: Grouping
    program: Program | None
    legal: bool
    total_us: float
    kernel_us: dict[str, float] = field(default_factory=dict)
    violations: list[str] = field(default_factory=list)
    error: str | None = None

    @property
    def total_cycles(self) -> float:  # reference field name; B200 costs are in microseconds
        return self.total_us

    def to_dict(self) -> dict[str, Any]:
        kernels = [] if self.program is None else [k.name for k in self.program.kernels]
        return dict(index=self.index, grouping=self.grouping, legal=self.legal, total_us=self.total_us,
                    kernel_us=self.kernel_us, kernels=kernels, violations=self.violations, error=self.error)


@dataclass
class PlanResult:
    best: Candidate
    candidates: list[Candidate]

    @property
    def program(self) -> Program:
        assert self.best.program is not None
        return self.best.program


# ------------------------------------------------------ set partitions (RGS)
def restricted_growth_strings(n: int) -> Iterator[tuple[int, ...]]:
    """Every RGS of length ``n`` in lexicographic order (Bell(n) of them):
    a[0] = 0 and a[i] <= 1 + max(a[:i])."""
    if n == 0:
        yield ()
        return
    a, peak = [0] * n, [0] * n  # peak[i] = max(a[:i+1])
    while True:
        yield tuple(a)
        i = n - 1
        while i > 0 and a[i] > peak[i - 1]:  # a[i] is already at its ceiling
            i -= 1
        if i == 0:
            return
        a[i] += 1
        peak[i] = max(peak[i - 1], a[i])
        for j in range(i + 1, n):
            a[j], peak[j] = 0, peak[i]


def set_partitions(items: Sequence[str]) -> list[list[list[str]]]:
    """All partitions of ``items`` into non-empty blocks (each block in item order)."""
    out = []
    for rgs in restricted_growth_strings(len(items)):
        blocks: list[list[str]] = [[] for _ in range(max(rgs, default=-1) + 1)]
        for item, label in zip(items, rgs):
            blocks[label].append(item)
        out.append(blocks)
    return out


def _options(members: list[str], mode: str) -> list[tuple[int, ...]]:
    """The RGS tried for one sibling set: all of them (exhaustive, up to six
    members), else all-merged and all-split."""
    n = len(members)
    if mode == "exhaustive" and n <= 6:
        return list(restricted_growth_strings(n))
    merged, split = (0,) * n, tuple(range(n))
    return [merged] if n == 1 else [merged, split]


def _grouping(sets: list[list[str]], choice: Sequence[tuple[int, ...]]) -> Grouping:
    """GEMM name -> kernel group id for one RGS per sibling set (ids unique across sets)."""
    grouping: Grouping = {}
    base = 0
    for members, rgs in zip(sets, choice):
        for m, label in zip(members, rgs):
            grouping[m] = base + label
        base += max(rgs, default=-1) + 1
    return grouping


def enumerate_groupings(g: OpGraph, mode: str = "exhaustive", max_candidates: int = 512) -> list[Grouping]:
    """Groupings of the exhaustive product (at most ``max_candidates``)."""
    sets = sibling_sets(g)
    space = itertools.product(*(_options(s, mode) for s in sets))
    return [_grouping(sets, c) for c in itertools.islice(space, max_candidates)]


# -------------------------------------------------------------------- costing
def kernel_signature(spec, tensors) -> str:
    """Structural key of a kernel: everything its cost depends on, nothing
    that names it (so equal layers share one cost evaluation)."""
    operands = tuple((a.role, a.name, tuple(tensors[a.tensor].shape), tuple(a.cols or ())) for a in spec.args)
    body = tuple((op.op, tuple(op.inputs), repr(sorted(op.attrs.items()))) for op in spec.epilogue)
    key = repr((spec.kind, sorted(spec.attrs.items(), key=lambda kv: kv[0]), spec.grid, spec.k_extent,
                tuple((gm.acc, gm.rhs) for gm in spec.gemms), bool(spec.sumsq), operands, body,
                tuple(o.value for o in spec.outputs)))
    return hashlib.sha1(key.encode()).hexdigest()


class _Coster:
    """Tile search + cost per kernel, memoised on :func:`kernel_signature`."""

    def __init__(self, hw: B200Spec, launch_us: float) -> None:
        self.hw, self.launch_us = hw, launch_us
        self.memo: dict[str, Any] = {}

    def __call__(self, program: Program) -> tuple[float, dict[str, float]]:
        per_kernel: dict[str, float] = {}
        for spec in program.kernels:
            sig = kernel_signature(spec, program.tensors)
            if sig not in self.memo:
                self.memo[sig] = search_tiles(spec, program.tensors, self.hw)
            found = self.memo[sig]
            spec.tiles = dict(found.best.tiles)
            spec.cost = {"us": found.best.us, "breakdown": found.best.to_dict(),
                         "alternatives": [{"tiles": r.tiles, "us": r.us} for r in found.top]}
            per_kernel[spec.name] = found.best.us
        return sum(per_kernel.values()) + self.launch_us * len(program.kernels), per_kernel


def cost_program(program: Program, hw: B200Spec, launch_us: float, memo: dict | None = None) -> tuple[float, dict[str, float]]:
    """Modelled forward time of ``program``: per-kernel costs plus one launch each."""
    coster = _Coster(hw, launch_us)
    if memo is not None:
        coster.memo = memo
    return coster(program)


# --------------------------------------------------------------------- search
class _Search:
    def __init__(self, g: OpGraph, name: str, coster: _Coster) -> None:
        self.g, self.name, self.coster = g, name, coster
        self.sets = sibling_sets(g)
        self.tried: dict[tuple, Candidate] = {}

    @property
    def candidates(self) -> list[Candidate]:
        return list(self.tried.values())

    def candidate(self, choice: Sequence[tuple[int, ...]]) -> Candidate:
        key = tuple(choice)
        if key in self.tried:
            return self.tried[key]
        grouping = _grouping(self.sets, choice)
        cand = Candidate(len(self.tried), grouping, None, False, float("inf"))
        try:
            cand.program = build_program(self.g, grouping, name=self.name)
            report = check_program(cand.program)
            if not report.ok:
                cand.violations = [str(v) for v in report.violations]
            else:
                cand.total_us, cand.kernel_us = self.coster(cand.program)
                cand.legal = True
        except (PartitionError, CostModelError) as e:
            cand.error = str(e)
        self.tried[key] = cand
        return cand


def _rank(c: Candidate) -> tuple[float, int]:
    return c.total_us, len(c.program.kernels) if c.program is not None else 1 << 30


def plan(g: OpGraph, hw: B200Spec, config, name: str = "program", max_candidates: int = 512) -> PlanResult:
    """The cheapest legal grouping: exhaustive over the product of the per-set
    options when it has at most ``max_candidates`` members, else coordinate
    descent (a sweep tries every option of every set with the others fixed;
    at most four sweeps, stopping early when one changes nothing)."""
    launch_us = float(getattr(config, "kernel_launch_overhead_us", hw.launch_us))
    search = _Search(g, name, _Coster(hw, launch_us))
    options = [_options(s, getattr(config, "planner_mode", "exhaustive")) for s in search.sets]
    space = 1
    for opts in options:
        space *= len(opts)
    exhaustive = space <= max_candidates
    if exhaustive:
        for choice in itertools.product(*options):
            search.candidate(choice)
    else:
        current = [opts[0] for opts in options]  # option 0 is all-merged
        best = search.candidate(current)
        for _sweep in range(4):
            improved = False
            for si, opts in enumerate(options):
                for opt in opts:
                    if opt == current[si]:
                        continue
                    trial = current[:si] + [opt] + current[si + 1:]
                    cand = search.candidate(trial)
                    if cand.legal and _rank(cand) < _rank(best):
                        best, current, improved = cand, trial, True
            if not improved:
                break
    cands = search.candidates
    legal = [c for c in cands if c.legal]
    if not legal:
        details = "\n".join(f"  candidate {c.index}: {c.error or c.violations}" for c in cands[:10])
        raise PartitionError(f"no legal partition among {len(cands)} candidates:\n{details}")
    best = min(legal, key=_rank)
    best.program.metadata["plan"] = {"candidates": len(cands), "legal": len(legal), "total_us": best.total_us,
                                     "kernel_us": best.kernel_us, "launch_us": launch_us,
                                     "search": "exhaustive" if exhaustive else "coordinate descent",
                                     "search_space": space}
    return PlanResult(best, cands)
