"""Run a compiled program from its results directory, without re-capture.

``compile_model(..., CompileConfig(save_params=True))`` leaves the chosen
OpIR Program (``06_opir.json``) and the transformed weights (``params.pt``)
in ``results_dir / run_name`` (the reference writes the same two files:
src/torch_helion/pipeline.py:100-107, src/torch_helion/optimizer/opir.py:141-169).
``load_compiled`` binds them to a GPU again: no FX capture, canonicalisation
or planning, the same th_* launch sequence, optionally replayed as one CUDA
graph.
"""

from __future__ import annotations

from pathlib import Path

import torch

from .optimizer.opir import Program


def load_compiled(run_dir: str | Path, device: str | torch.device = "cuda", cuda_graph: bool = False):
    """The device program saved in ``run_dir``, ready to call: ``mod(x)`` returns the outputs."""
    from .b200.runtime import CompiledProgram

    run_dir = Path(run_dir)
    opir, weights = run_dir / "06_opir.json", run_dir / "params.pt"
    if not opir.exists() or not weights.exists():
        raise FileNotFoundError(f"{run_dir} lacks 06_opir.json / params.pt (compile with CompileConfig(save_params=True))")
    program = Program.from_json(opir)
    params = torch.load(weights, map_location="cpu", weights_only=True)
    missing = [n for n in program.params if n not in params]
    if missing:
        raise KeyError(f"params.pt lacks {missing[:4]}")
    mod = CompiledProgram(program, params, device)
    if cuda_graph:
        mod.capture_graph()
    return mod
