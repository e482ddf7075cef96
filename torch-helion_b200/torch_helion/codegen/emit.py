"""Codegen artefacts: the per-kernel B200 launch plan.

The reference's ``emit_program(program, config, out_dir) -> {name: Path}``
writes one generated Helion module per kernel (src/torch_helion/codegen/
emit.py:500-520).  The B200 backend does not generate code -- every
KernelSpec maps onto a hand-written sm_100a kernel -- so the same entry
point writes, per kernel, the lowered ``th_*`` launch plan as JSON
(segments, fused epilogue stages, tiles, modelled cost).  Kernels that
cannot be lowered raise :class:`CodegenError`.
"""

from __future__ import annotations

import json
from dataclasses import asdict, is_dataclass
from pathlib import Path
from typing import Any

from ..optimizer.opir import KernelSpec, Program


class CodegenError(RuntimeError):
    pass


ENTRY_POINTS = {"gemm": "th_gemm", "attention": "th_attention", "ssd": "th_ssd", "causal_conv1d": "th_conv1d",
                "rmsnorm": "th_rmsnorm", "embedding": "th_embedding"}


def _plain(o: Any) -> Any:
    if is_dataclass(o):
        return {k: _plain(v) for k, v in asdict(o).items()}
    if isinstance(o, dict):
        return {str(k): _plain(v) for k, v in o.items()}
    if isinstance(o, (list, tuple)):
        return [_plain(v) for v in o]
    return o


def launch_plan(spec: KernelSpec, program: Program) -> dict[str, Any]:
    from ..b200.lower import LoweringError, lower_kernel

    try:
        plan = lower_kernel(spec, program)
    except LoweringError as e:
        raise CodegenError(str(e)) from e
    d = {"kernel": spec.name, "kind": spec.kind, "entry_point": ENTRY_POINTS[spec.kind], "plan": _plain(plan),
         "tiles": spec.tiles, "modelled_us": spec.cost.get("us")}
    if spec.kind == "gemm":
        d["extra_launches"] = ["th_rowstat (when no producer provides the row statistics)"] if spec.sumsq else []
    return d


def emit_program(program: Program, config, out_dir: Path) -> dict[str, Path]:
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    written: dict[str, Path] = {}
    for spec in program.kernels:
        p = out_dir / f"{spec.name}.json"
        p.write_text(json.dumps(launch_plan(spec, program), indent=2, default=str))
        written[spec.name] = p
    return written
