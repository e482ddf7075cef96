"""Kernel legality for the B200 backend.

The reference checks Loom's constraints C2-C5 (one reduction loop,
32-aligned extents, registered ops, src/torch_helion/optimizer/
legality.py:56-138).  On B200 a kernel is legal when it lowers to a
``th_*`` launch: the epilogue matches th_gemm's fused stages, row strides
are 16-byte multiples for TMA, rope/SwiGLU segments line up with the
tile, and the macro kernels were built for the shape.  The single source
of truth is :func:`torch_helion.b200.lower.check_lowering`.
"""

from __future__ import annotations

from dataclasses import dataclass, field

from .opir import Program


@dataclass
class Violation:
    kernel: str
    rule: str
    message: str

    def __str__(self) -> str:
        return f"[{self.kernel}] {self.rule}: {self.message}"


@dataclass
class LegalityReport:
    violations: list[Violation] = field(default_factory=list)

    @property
    def ok(self) -> bool:
        return not self.violations

    def __str__(self) -> str:
        return "legal" if self.ok else "\n".join(str(v) for v in self.violations)


def check_program(program: Program) -> LegalityReport:
    from ..b200.lower import check_lowering

    rep = LegalityReport()
    for msg in check_lowering(program):
        kname = msg.split(":", 1)[0]
        rep.violations.append(Violation(kname, "b200", msg))
    return rep
