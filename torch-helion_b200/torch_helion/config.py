"""Compile-time configuration (the reference's ``CompileConfig``, config.py:15-66,
with the B200 backend knobs added; every reference field is kept)."""

from __future__ import annotations

import os
from dataclasses import dataclass, field
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parents[1]      # torch-helion_b200/
REPO_ROOT = PKG_ROOT.parent
DEFAULT_HW_SPEC = REPO_ROOT / "MEASURED_PEAKS.json"
DEFAULT_RESULTS_DIR = REPO_ROOT / "results"


@dataclass
class CompileConfig:
    """Knobs of :func:`torch_helion.compile_model`.

    Reference fields (same meaning): ``run_name``, ``hw_spec`` (here: the
    B200 peaks file; missing -> nominal B200 figures), ``results_dir``,
    ``planner_mode`` ("exhaustive" | "greedy"), ``tile_alignment``,
    ``max_tile``, ``kernel_launch_overhead`` (reference unit: cycles; kept
    for compatibility), ``verify_with_loom`` / ``loom_njobs`` /
    ``loom_topk_candidates`` / ``check_frontend`` / ``validate_workers``
    (Loom-only; accepted and ignored by the B200 backend), ``save_params``,
    ``dtype``.

    B200 fields:
      backend            "b200" (the only backend of this package)
      device             CUDA device the compiled module runs on
      execute            build the device program and run the reference check
                         (False: compile only, no GPU needed)
      verify_passes      re-evaluate the graph after every canonicalisation pass
      reference_check    compare the B200 output with the eager model
      tolerance          reference-check bound (max relative error)
      cuda_graph         replay the forward as one CUDA graph
      kernel_launch_overhead_us  per-kernel launch cost in the planner (us)
      world_size / tp_mode  tensor parallelism ("heads" for the Llama block)
      tp_chunks          row chunks of the tensor-parallel part after attention:
                         each chunk's all-reduce overlaps the next chunk's GEMMs
      tp_comm_sms        SMs the GEMMs of that overlapped part leave to the collectives
                         (also the grid of the multicast all-reduce kernel); None: 16 with
                         the multicast all-reduce, 0 with NCCL
      tp_allreduce       "multimem" (th_allreduce on symmetric buffers through NVSwitch
                         multicast), "nccl", or "auto" (multimem where every rank supports it)
      measure_iters      time the forward on the device (0 = skip)
    """

    run_name: str = "run"
    hw_spec: Path = field(default_factory=lambda: Path(os.environ.get("TORCH_HELION_HW_SPEC", DEFAULT_HW_SPEC)))
    results_dir: Path = field(default_factory=lambda: Path(os.environ.get("TORCH_HELION_RESULTS", DEFAULT_RESULTS_DIR)))
    planner_mode: str = "exhaustive"
    tile_alignment: int = 32
    max_tile: int = 512
    kernel_launch_overhead: float = 2000.0
    verify_with_loom: bool = False
    loom_njobs: int = 8
    loom_topk_candidates: int = 1
    check_frontend: bool = False
    validate_workers: int = 4
    save_params: bool = False
    dtype: str = "float16"
    # --- B200
    backend: str = "b200"
    device: str = "cuda"
    execute: bool = True
    verify_passes: bool = True
    reference_check: bool = True
    tolerance: float = 2e-2
    cuda_graph: bool = False
    kernel_launch_overhead_us: float = 3.0
    world_size: int = 1
    tp_mode: str | None = None
    tp_chunks: int = 4
    tp_comm_sms: int | None = None
    tp_allreduce: str = "auto"
    measure_iters: int = 0

    @property
    def run_dir(self) -> Path:
        return Path(self.results_dir) / self.run_name

    def hw_spec_dir(self) -> Path:
        return Path(self.hw_spec).resolve().parent
