"""Layout provenance: which element of a base tensor does a view read?

ATen states head splits, transposes and broadcasts as chains of ``view`` /
``permute`` / ``expand`` / ``clone`` / ``slice`` / ``cast`` nodes.  Like the
reference (src/torch_helion/optimizer/layout.py:61-128) we answer pattern
questions ("is this a [B,H,S,d] head split of a token-major [T, H*d]
tensor?") by replaying the chain instead of reasoning about strides.  The
reference replays it on a full ``arange`` index tensor, which is the size of
the activation (a gigabyte of int64 at Llama-8B shapes); here the chain is
replayed backwards on a fixed set of probe *coordinates* (all corners of
the view plus seeded random points), which costs O(probes x chain) at any
size.  A pattern matches when every probe lands where the pattern says.
"""

from __future__ import annotations

import itertools
import math
from dataclasses import dataclass

import torch

from ..capture.opgraph import OpGraph, OpNode

TRACEABLE = ("view", "permute", "expand", "clone", "slice", "cast")
_N_RANDOM_PROBES = 192


def _ravel(c: torch.Tensor, shape) -> torch.Tensor:
    flat = torch.zeros(c.shape[0], dtype=torch.int64)
    for j, s in enumerate(shape):
        flat = flat * int(s) + c[:, j]
    return flat


def _unravel(flat: torch.Tensor, shape) -> torch.Tensor:
    out = torch.empty(flat.shape[0], len(shape), dtype=torch.int64)
    rem = flat.clone()
    for j in range(len(shape) - 1, -1, -1):
        s = int(shape[j])
        out[:, j] = rem % s
        rem = rem // s
    return out


@dataclass
class Provenance:
    base: str
    base_shape: tuple[int, ...]
    shape: tuple[int, ...]
    chain: list[str]  # layout node names, base-first
    _nodes: list[OpNode]
    _in_shapes: list[tuple[int, ...]]

    # ---- coordinate replay
    def to_base(self, coords: torch.Tensor) -> torch.Tensor:
        """Flat base index read by each view coordinate ``coords [K, rank]``."""
        c = coords
        for node, ins in zip(reversed(self._nodes), reversed(self._in_shapes)):
            out_shape = node.type.shape
            if node.op == "view":
                c = _unravel(_ravel(c, out_shape), ins)
            elif node.op == "permute":
                nc = torch.empty(c.shape[0], len(ins), dtype=torch.int64)
                for j, d in enumerate(node.attrs["dims"]):
                    nc[:, d] = c[:, j]
                c = nc
            elif node.op == "expand":
                lead = len(out_shape) - len(ins)
                c = c[:, lead:].clone()
                for j, s in enumerate(ins):
                    if s == 1:
                        c[:, j] = 0
            elif node.op == "slice":
                c = c.clone()
                c[:, node.attrs["dim"]] += node.attrs["start"]
            # clone / cast: identity
        return _ravel(c, self.base_shape)

    def probes(self) -> torch.Tensor:
        return probe_coords(self.shape)

    @property
    def numel(self) -> int:
        return math.prod(self.shape) if self.shape else 1

    def is_identity_reshape(self) -> bool:
        if self.numel != (math.prod(self.base_shape) if self.base_shape else 1):
            return False
        if not self.chain:
            return True
        p = self.probes()
        return bool(torch.equal(self.to_base(p), _ravel(p, self.shape)))

    def matches(self, expected_fn) -> bool:
        """``expected_fn(coords) -> flat base index`` agrees on every probe."""
        p = self.probes()
        return bool(torch.equal(self.to_base(p), expected_fn(p)))


def probe_coords(shape) -> torch.Tensor:
    shape = tuple(int(s) for s in shape)
    if not shape:
        return torch.zeros(1, 0, dtype=torch.int64)
    per_dim = [sorted({0, s - 1, s // 2, min(1, s - 1)}) for s in shape]
    corners = list(itertools.islice(itertools.product(*per_dim), 512))
    g = torch.Generator().manual_seed(1234)
    rnd = torch.stack([torch.randint(0, s, (_N_RANDOM_PROBES,), generator=g) for s in shape], 1)
    return torch.cat((torch.tensor(corners, dtype=torch.int64).reshape(-1, len(shape)), rnd), 0)


def trace_layout(graph: OpGraph, name: str) -> Provenance:
    chain: list[OpNode] = []
    cur = graph[name]
    while cur.kind == "layout" and cur.op in TRACEABLE and len(cur.inputs) == 1:
        chain.append(cur)
        cur = graph[cur.inputs[0]]
    chain.reverse()
    in_shapes = [graph[n.inputs[0]].type.shape for n in chain]
    return Provenance(cur.name, cur.type.shape, graph[name].type.shape, [n.name for n in chain], chain, in_shapes)


def _divisors(n: int) -> list[int]:
    return [d for d in range(1, n + 1) if n % d == 0]


def head_split_fn(b: int, s: int, h: int, d: int, kv: int, transpose_last: bool = False, merged: bool = False):
    """Expected flat index of a [B,H,S,d] (or [B*H,S,d]; ``transpose_last``:
    last two swapped) head-split view of a token-major [B*S, kv*d] base in
    which query head ``i`` reads kv head ``i // (H/kv)``."""
    rep = h // kv

    def fn(c: torch.Tensor) -> torch.Tensor:
        if merged:
            bh, x1, x2 = c[:, 0], c[:, 1], c[:, 2]
            bi, hi = bh // h, bh % h
        else:
            bi, hi, x1, x2 = c[:, 0], c[:, 1], c[:, 2], c[:, 3]
        si, di = (x2, x1) if transpose_last else (x1, x2)
        return (bi * s + si) * (kv * d) + (hi // rep) * d + di

    return fn


def match_head_split(prov: Provenance, transpose_last: bool = False) -> dict | None:
    """``{batch, seq, heads, head_dim, kv_heads}`` when ``prov`` is a head
    split of a token-major base (grouped KV heads allowed), else None."""
    shape = prov.shape
    base_numel = math.prod(prov.base_shape)
    cands: list[tuple[int, int, int, int, bool]] = []
    if len(shape) == 4:
        b, h = shape[0], shape[1]
        s, d = (shape[3], shape[2]) if transpose_last else (shape[2], shape[3])
        cands.append((b, h, s, d, False))
    elif len(shape) == 3:
        bh = shape[0]
        s, d = (shape[2], shape[1]) if transpose_last else (shape[1], shape[2])
        for b in _divisors(bh):
            cands.append((b, bh // b, s, d, True))
    for b, h, s, d, merged in cands:
        for kv in sorted(_divisors(h), reverse=True):
            if b * s * kv * d != base_numel:
                continue
            if prov.matches(head_split_fn(b, s, h, d, kv, transpose_last, merged)):
                return {"batch": b, "seq": s, "heads": h, "head_dim": d, "kv_heads": kv}
    return None


def head_merge_fn(b: int, s: int, h: int, d: int):
    """Expected flat index (into the attention output viewed [B*H, S, d] or
    [B, H, S, d]) of the token-major [B*S, H*d] merge."""

    def fn(c: torch.Tensor) -> torch.Tensor:
        t, f = c[:, 0], c[:, 1]
        bi, si = t // s, t % s
        hi, di = f // d, f % d
        return ((bi * h + hi) * s + si) * d + di

    return fn


def column_slice(prov: Provenance) -> tuple[int, int] | None:
    """(start, end) when the view is a contiguous column range of a 2-D (or
    [B, S, F]) base with the same leading extent, else None."""
    bs, vs = prov.base_shape, prov.shape
    if len(bs) < 2 or len(vs) < 2 or math.prod(bs[:-1]) != math.prod(vs[:-1]):
        return None
    F_in, F_out = bs[-1], vs[-1]
    p = prov.probes()
    got = prov.to_base(p)
    rows = _ravel(p[:, :-1], vs[:-1]) if len(vs) > 1 else torch.zeros(p.shape[0], dtype=torch.int64)
    start = int(got[0] - rows[0] * F_in - p[0, -1])
    if start < 0 or start + F_out > F_in:
        return None
    if torch.equal(got, rows * F_in + start + p[:, -1]):
        return (start, start + F_out)
    return None
