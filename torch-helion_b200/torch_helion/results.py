"""The results directory of one compilation.

The artefact names are the reference's (src/torch_helion/results.py:1-23) so
tools that browse a reference run find the same files; the B200 backend adds
its own (launch plans, measurements) and records every file it writes in a
manifest:

    results/<run_name>/
      00_model.txt                 model repr and configuration
      01_fx_graph.txt              exported ATen graph
      01_fx_op_histogram.json
      02_opgraph_raw.{json,txt}    OpGraph straight from the FX graph
      03_opgraph_canonical.{json,txt}, 03_pass_log.json
      04_hw_spec.json              B200 peaks used by the cost model
      05_plan/candidates.json, 05_plan/plan.md
      06_opir.{json,txt}           the chosen Program
      07_launch_plan.json          every kernel's th_* launch (lowered plan)
      08_reference_check.json      B200 output vs the eager model
      09_cost_report.{md,json}     modelled vs measured cost per kernel
      10_measured.json             (measure_iters > 0) device-timed forward
      kernels/<kernel>.json        per-kernel launch plan
      params.pt                    (save_params) transformed weights
      timings.json                 wall time per stage
      manifest.json                every artefact above: stage, bytes
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Any


class _ArtefactEncoder(json.JSONEncoder):
    """JSON for the pipeline's objects: anything with ``to_dict``, paths and
    sets; the rest falls back to ``str`` so an artefact never fails to write."""

    def default(self, o: Any) -> Any:  # noqa: D401 - json hook
        to_dict = getattr(o, "to_dict", None)
        if callable(to_dict):
            return to_dict()
        if isinstance(o, (set, frozenset, tuple)):
            return list(o)
        return str(o)


@dataclass
class Artefact:
    name: str
    stage: str
    bytes: int


class RunDirectory:
    """Writes the artefacts of one run under ``run_dir``.

    Text and JSON artefacts are written to a temporary name and renamed into
    place, so a reader never sees a half-written file; ``reserve`` hands out a
    path for artefacts another library writes (``torch.save``, the OpGraph's
    own JSON writer).  ``stage`` labels what follows in the manifest."""

    def __init__(self, run_dir: Path) -> None:
        self.run_dir = Path(run_dir)
        self.run_dir.mkdir(parents=True, exist_ok=True)
        self.stage = "setup"
        self._written: dict[str, str] = {}

    def reserve(self, name: str) -> Path:
        target = self.run_dir / name
        target.parent.mkdir(parents=True, exist_ok=True)
        self._written[name] = self.stage
        return target

    # the reference writer's name for ``reserve``
    path = reserve

    def write_text(self, name: str, text: str) -> Path:
        target = self.reserve(name)
        tmp = target.with_name(f".{target.name}.{os.getpid()}.tmp")
        tmp.write_text(text)
        tmp.replace(target)
        return target

    def write_json(self, name: str, obj: Any) -> Path:
        return self.write_text(name, json.dumps(obj, indent=2, cls=_ArtefactEncoder))

    def artefacts(self) -> list[Artefact]:
        out = []
        for name, stage in sorted(self._written.items()):
            f = self.run_dir / name
            if f.is_file():
                out.append(Artefact(name, stage, f.stat().st_size))
            elif f.is_dir():
                for g in sorted(p for p in f.rglob("*") if p.is_file()):
                    out.append(Artefact(str(g.relative_to(self.run_dir)), stage, g.stat().st_size))
        return out

    def write_manifest(self) -> Path:
        return self.write_json("manifest.json", [a.__dict__ for a in self.artefacts()])

    def listing(self) -> list[str]:
        return sorted(str(p.relative_to(self.run_dir)) for p in self.run_dir.rglob("*")
                      if p.is_file() and not p.name.startswith("."))


ResultsWriter = RunDirectory

__all__ = ["RunDirectory", "ResultsWriter", "Artefact"]
