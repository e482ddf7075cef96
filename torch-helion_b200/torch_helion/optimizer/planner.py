"""Planner: choose which sibling GEMMs share a kernel, by the B200 cost model.

Same search as the reference planner (src/torch_helion/optimizer/
planner.py:70-164): every set partition of each sibling set (Bell-number
many, ``exhaustive``) or just all-merged / all-split (``greedy``); each
candidate is partitioned, checked for legality, costed kernel by kernel
(memoised on a structural signature) plus a launch overhead per kernel,
and the cheapest legal program wins.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from itertools import product
from typing import Any

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
        return {"index": self.index, "grouping": self.grouping, "legal": self.legal, "total_us": self.total_us,
                "kernel_us": self.kernel_us, "kernels": [k.name for k in self.program.kernels] if self.program else [],
                "violations": self.violations, "error": self.error}


@dataclass
class PlanResult:
    best: Candidate
    candidates: list[Candidate]

    @property
    def program(self) -> Program:
        assert self.best.program is not None
        return self.best.program


def set_partitions(items: list[str]) -> list[list[list[str]]]:
    if not items:
        return [[]]
    first, rest = items[0], items[1:]
    out = []
    for part in set_partitions(rest):
        out.append([[first]] + part)
        for i in range(len(part)):
            out.append(part[:i] + [[first] + part[i]] + part[i + 1:])
    return out


def _per_set_partitions(g: OpGraph, mode: str) -> list[list[list[list[str]]]]:
    per_set = []
    for s in sibling_sets(g):
        if mode == "exhaustive" and len(s) <= 6:
            per_set.append(set_partitions(s))
        else:
            per_set.append([[list(s)], [[m] for m in s]] if len(s) > 1 else [[list(s)]])
    return per_set


def _grouping(combo) -> Grouping:
    grouping: Grouping = {}
    gid = 0
    for part in combo:
        for block in part:
            for m in block:
                grouping[m] = gid
            gid += 1
    return grouping


def enumerate_groupings(g: OpGraph, mode: str = "exhaustive", max_candidates: int = 512) -> list[Grouping]:
    """The full product of the per-set partitions (at most ``max_candidates``)."""
    groupings: list[Grouping] = []
    for combo in product(*_per_set_partitions(g, mode)):
        groupings.append(_grouping(combo))
        if len(groupings) >= max_candidates:
            break
    return groupings


def kernel_signature(spec, tensors) -> str:
    d = spec.to_dict()
    for k in ("name", "tiles", "cost"):
        d.pop(k, None)
    d["shapes"] = {a.name: list(tensors[a.tensor].shape) for a in spec.args}
    d["args"] = [[a.name, a.role, a.cols] for a in spec.args]
    d["outputs"] = [o.value for o in spec.outputs]
    return json.dumps(d, sort_keys=True, default=str)


def cost_program(program: Program, hw: B200Spec, launch_us: float, memo: dict | None = None) -> tuple[float, dict[str, float]]:
    total, per = 0.0, {}
    memo = memo if memo is not None else {}
    for spec in program.kernels:
        key = kernel_signature(spec, program.tensors)
        res = memo.get(key)
        if res is None:
            res = search_tiles(spec, program.tensors, hw)
            memo[key] = res
        spec.tiles = dict(res.best.tiles)
        spec.cost = {"us": res.best.us, "breakdown": res.best.to_dict(), "alternatives": [
            {"tiles": r.tiles, "us": r.us} for r in res.top]}
        per[spec.name] = res.best.us
        total += res.best.us + launch_us
    return total, per


def plan(g: OpGraph, hw: B200Spec, config, name: str = "program", max_candidates: int = 512) -> PlanResult:
    """Cheapest legal grouping.  The whole product of the per-set partitions
    is searched when it has at most ``max_candidates`` members; otherwise
    (deep models: one sibling set per layer and projection) coordinate
    descent over the sets, starting from all-merged, each set trying all its
    partitions with the others fixed, until a sweep changes nothing.  The
    cost is a sum over kernels and a set's grouping changes only its own
    kernels, so the descent reaches the same optimum."""
    launch_us = float(getattr(config, "kernel_launch_overhead_us", hw.launch_us))
    per_set = _per_set_partitions(g, getattr(config, "planner_mode", "exhaustive"))
    cands: list[Candidate] = []
    memo: dict[str, Any] = {}
    seen: dict[str, Candidate] = {}

    def evaluate(combo) -> Candidate:
        grouping = _grouping(combo)
        key = json.dumps(grouping, sort_keys=True)
        if key in seen:
            return seen[key]
        i = len(cands)
        try:
            program = build_program(g, grouping, name=name)
        except PartitionError as e:
            c = Candidate(i, grouping, None, False, float("inf"), error=str(e))
        else:
            rep = check_program(program)
            if not rep.ok:
                c = Candidate(i, grouping, program, False, float("inf"), violations=[str(v) for v in rep.violations])
            else:
                try:
                    total, per = cost_program(program, hw, launch_us, memo)
                    c = Candidate(i, grouping, program, True, total, per)
                except CostModelError as e:
                    c = Candidate(i, grouping, program, False, float("inf"), error=str(e))
        cands.append(c)
        seen[key] = c
        return c

    rank = lambda c: (c.total_us, len(c.program.kernels) if c.program else 1 << 30)
    n_product = 1
    for p in per_set:
        n_product *= len(p)
    if n_product <= max_candidates:
        for combo in product(*per_set):
            evaluate(combo)
    else:
        combo = [p[0] if len(p[0]) == 1 else next(q for q in p if len(q) == 1) for p in per_set]  # all merged
        best = evaluate(combo)
        for _ in range(4):
            changed = False
            for si, options in enumerate(per_set):
                for opt in options:
                    if opt is combo[si]:
                        continue
                    trial = list(combo)
                    trial[si] = opt
                    c = evaluate(trial)
                    if c.legal and rank(c) < rank(best):
                        best, combo, changed = c, trial, True
            if not changed:
                break
    legal = [c for c in cands if c.legal]
    if not legal:
        details = "\n".join(f"  candidate {c.index}: {c.error or c.violations}" for c in cands[:10])
        raise PartitionError(f"no legal partition among {len(cands)} candidates:\n{details}")
    best = min(legal, key=rank)
    best.program.metadata["plan"] = {"candidates": len(cands), "legal": len(legal), "total_us": best.total_us,
                                     "kernel_us": best.kernel_us, "launch_us": launch_us,
                                     "search": "exhaustive" if n_product <= max_candidates else "coordinate descent",
                                     "search_space": n_product}
    return PlanResult(best, cands)
