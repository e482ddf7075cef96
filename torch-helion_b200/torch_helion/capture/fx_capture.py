"""PyTorch model -> core-ATen FX graph with static shapes (torch.export).

Behaviour of the reference capture (src/torch_helion/capture/fx_capture.py:37-50):
``torch.export.export`` with the example arguments, parameters and buffers
lifted to graph inputs, then ``run_decompositions()`` down to core ATen.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Sequence

import torch
from torch.export import ExportedProgram


@dataclass
class CapturedFx:
    exported: ExportedProgram
    example_args: tuple[Any, ...]

    @property
    def graph_module(self) -> torch.fx.GraphModule:
        return self.exported.graph_module

    def text(self) -> str:
        return self.graph_module.graph.python_code("self").src

    def op_histogram(self) -> dict[str, int]:
        hist: dict[str, int] = {}
        for n in self.graph_module.graph.nodes:
            if n.op == "call_function":
                hist[str(n.target)] = hist.get(str(n.target), 0) + 1
        return dict(sorted(hist.items()))


def export_to_fx(model: torch.nn.Module, example_args: Sequence[Any]) -> CapturedFx:
    model = model.eval()
    args = tuple(example_args)
    with torch.no_grad():
        ep = torch.export.export(model, args)
        ep = ep.run_decompositions()
    return CapturedFx(exported=ep, example_args=args)
