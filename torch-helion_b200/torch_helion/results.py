"""Results directory of one compilation (layout of the reference's
results.py:1-23, with the B200 artefacts):

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
      09_cost_report.{md,json}     modelled cost per kernel
      10_measured.json             (measure_iters > 0) device-timed forward
      kernels/<kernel>.json        per-kernel launch plan
      params.pt                    (save_params) transformed weights
      timings.json                 wall time per stage
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any


class ResultsWriter:
    def __init__(self, run_dir: Path) -> None:
        self.run_dir = Path(run_dir)
        self.run_dir.mkdir(parents=True, exist_ok=True)
        self.files: list[Path] = []

    def path(self, name: str) -> Path:
        p = self.run_dir / name
        p.parent.mkdir(parents=True, exist_ok=True)
        return p

    def write_text(self, name: str, text: str) -> Path:
        p = self.path(name)
        p.write_text(text)
        self.files.append(p)
        return p

    def write_json(self, name: str, obj: Any) -> Path:
        return self.write_text(name, json.dumps(obj, indent=2, default=_default))

    def listing(self) -> list[str]:
        return sorted(str(p.relative_to(self.run_dir)) for p in self.run_dir.rglob("*") if p.is_file())


def _default(o: Any) -> Any:
    if hasattr(o, "to_dict"):
        return o.to_dict()
    if isinstance(o, Path):
        return str(o)
    if isinstance(o, (set, tuple)):
        return list(o)
    return str(o)
