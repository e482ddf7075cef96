"""End-to-end pipeline: PyTorch model -> OpGraph -> OpIR -> sm_100a kernels.

::

    from torch_helion import compile_model, CompileConfig
    res = compile_model(model, example_args, CompileConfig(run_name="llama_block"))
    out = res.run(*inputs)            # forward on the B200
    print(res.program.summary())

The stages and their artefacts follow the reference pipeline
(src/torch_helion/pipeline.py:60-145): capture, canonicalise (numerically
verified pass by pass), plan (partition + cost model), codegen artefacts,
a reference check against the eager model, cost reports, timings.  The
B200 backend replaces Helion/Loom emission and validation with a device
program (:class:`torch_helion.b200.runtime.CompiledProgram`) built from the
hand-written kernels, and adds an optional device-timed measurement.
"""

from __future__ import annotations

import copy
import logging
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Sequence

import torch

from .capture import CapturedFx, OpGraph, capture
from .codegen.emit import emit_program
from .config import CompileConfig
from .cost_models.b200 import B200Spec
from .optimizer.evaluate import max_rel_err, rel_l2
from .optimizer.legality import check_program
from .optimizer.opir import Program
from .optimizer.passes import canonicalize
from .optimizer.planner import PlanResult, plan
from .results import RunDirectory

log = logging.getLogger("torch_helion")


@dataclass
class CompileResult:
    config: CompileConfig
    run_dir: Path
    fx: CapturedFx
    raw_graph: OpGraph
    graph: OpGraph
    hw: B200Spec
    plan: PlanResult
    program: Program
    kernel_files: dict[str, Path]
    validation: dict[str, Any] = field(default_factory=dict)
    reference_check: dict[str, Any] = field(default_factory=dict)
    loom_results: dict[str, Any] = field(default_factory=dict)
    timings: dict[str, float] = field(default_factory=dict)
    module: Any = None
    measured: dict[str, Any] = field(default_factory=dict)

    @property
    def estimated_us(self) -> float:
        return self.program.metadata.get("plan", {}).get("total_us", float("nan"))

    @property
    def estimated_cycles(self) -> float:
        """Reference name; the B200 model estimates microseconds."""
        return self.estimated_us

    def run(self, *inputs: torch.Tensor) -> list[torch.Tensor]:
        """Run the compiled forward on the GPU (inputs on CPU or GPU); returns device tensors."""
        if self.module is None:
            self.module = device_module(self.program, self.graph.params, self.config)
        return self.module(*inputs)

    def streaming_runner(self, depth: int = 2, cuda_graph: bool | None = None):
        """Overlapped serving from pinned host memory.  One GPU: a
        :class:`~torch_helion.b200.runtime.StreamingRunner` (host batches in,
        host outputs out, copies overlapped with the forward).  Tensor
        parallel (``world_size > 1``): a
        :class:`~torch_helion.b200.runtime.ShardedStreamingRunner` on this
        rank's module, each rank moving only its own rows over the host link."""
        from .b200.runtime import ShardedStreamingRunner, StreamingRunner

        if self.config.world_size > 1:
            if self.module is None:
                self.module = device_module(self.program, self.graph.params, self.config)
            return ShardedStreamingRunner(self.module, depth=depth)
        cg = self.config.cuda_graph if cuda_graph is None else cuda_graph
        return StreamingRunner(self.program, self.graph.params, self.config.device, depth=depth, cuda_graph=cg)


def device_module(program: Program, params: dict[str, torch.Tensor], config: CompileConfig):
    """The device program for ``config``: one GPU, or this rank's tensor-parallel
    shard when ``world_size > 1`` (``torch.distributed`` initialised, NCCL)."""
    from .b200.runtime import CompiledProgram

    if config.world_size <= 1:
        return CompiledProgram(program, params, config.device)
    import torch.distributed as dist

    from .b200.tp import shard_program

    if config.tp_mode not in (None, "heads"):
        raise ValueError(f"unknown tp_mode {config.tp_mode!r} (supported: 'heads')")
    if not dist.is_initialized() or dist.get_world_size() != config.world_size:
        raise RuntimeError(f"world_size={config.world_size} needs an initialised process group of that size")
    rank = dist.get_rank()
    sharded, sparams = shard_program(program, params, config.world_size, rank)
    return CompiledProgram(sharded, sparams, config.device, tp_rank=rank, tp_world=config.world_size,
                           allreduce=lambda t: dist.all_reduce(t), tp_chunks=config.tp_chunks,
                           tp_comm_sms=config.tp_comm_sms, tp_allreduce=config.tp_allreduce)


class _Stage:
    """Times one pipeline stage and labels the artefacts it writes."""

    def __init__(self, timings: dict[str, float], name: str, rundir: RunDirectory | None = None) -> None:
        self.timings, self.name, self.rundir = timings, name, rundir

    def __enter__(self) -> None:
        self.t0 = time.perf_counter()
        if self.rundir is not None:
            self.rundir.stage = self.name
        log.info("stage %s", self.name)

    def __exit__(self, *exc) -> None:
        self.timings[self.name] = time.perf_counter() - self.t0


def compile_model(model: torch.nn.Module, example_args: Sequence[Any], config: CompileConfig | None = None) -> CompileResult:
    config = config or CompileConfig()
    if config.backend != "b200":
        raise ValueError(f"unknown backend {config.backend!r} (this package implements 'b200')")
    rw = RunDirectory(config.run_dir)
    timings: dict[str, float] = {}

    with _Stage(timings, "capture", rw):
        fx, raw = capture(model, example_args)
        rw.write_text("00_model.txt", f"{model!r}\n\nconfig: {config!r}\n")
        rw.write_text("01_fx_graph.txt", fx.text())
        rw.write_json("01_fx_op_histogram.json", fx.op_histogram())
        raw.to_json(rw.path("02_opgraph_raw.json"))
        rw.write_text("02_opgraph_raw.txt", raw.summary())

    with _Stage(timings, "canonicalize", rw):
        graph, pass_log = canonicalize(raw, verify_inputs=list(example_args) if config.verify_passes else None)
        graph.to_json(rw.path("03_opgraph_canonical.json"))
        rw.write_text("03_opgraph_canonical.txt", graph.summary())
        rw.write_json("03_pass_log.json", pass_log)

    with _Stage(timings, "plan", rw):
        hw = B200Spec.load(config.hw_spec)
        rw.write_json("04_hw_spec.json", hw.summary())
        result = plan(graph, hw, config, name=config.run_name)
        program = result.program
        rw.write_json("05_plan/candidates.json", [c.to_dict() for c in result.candidates])
        rw.write_text("05_plan/plan.md", plan_report(result, hw, config))
        program.to_json(rw.path("06_opir.json"))
        rw.write_text("06_opir.txt", program.summary())

    with _Stage(timings, "codegen", rw):
        kernel_files = emit_program(program, config, rw.path("kernels"))
        rw.write_json("07_launch_plan.json", {k: str(v) for k, v in kernel_files.items()})
        if config.save_params:
            torch.save({n: graph.params[n] for n in program.params}, rw.path("params.pt"))

    res = CompileResult(config, rw.run_dir, fx, raw, graph, hw, result, program, kernel_files, timings=timings)

    if config.execute:
        with _Stage(timings, "build_device_program", rw):
            res.module = device_module(program, graph.params, config)
            if config.cuda_graph:
                res.module.capture_graph()
        if config.reference_check:
            with _Stage(timings, "reference_check", rw):
                res.reference_check = reference_check(model, example_args, res, config.tolerance)
                rw.write_json("08_reference_check.json", res.reference_check)
        if config.measure_iters > 0:
            with _Stage(timings, "measure", rw):
                res.measured = measure(res, example_args, config.measure_iters)
                rw.write_json("10_measured.json", res.measured)

    rw.write_json("09_cost_report.json", cost_report_json(program, hw, config))
    rw.write_text("09_cost_report.md", cost_report_md(program, hw, config, res.measured))
    rw.stage = "report"
    rw.write_json("timings.json", timings)
    rw.write_manifest()
    return res


def reference_check(model, example_args, res: CompileResult, tolerance: float) -> dict[str, Any]:
    """B200 output vs the eager model.  For low-precision models the primary
    comparison is the eager forward in fp32 on the model's (rounded)
    weights; the eager low-precision forward is recorded beside it."""
    outs = [o.float().cpu() for o in res.run(*example_args)]
    with torch.no_grad():
        ref = model(*example_args)
        refs = ref if isinstance(ref, (list, tuple)) else [ref]
        low = any(r.dtype in (torch.bfloat16, torch.float16) for r in refs)
        if low:
            m32 = copy.deepcopy(model).float()
            args32 = [a.float() if torch.is_tensor(a) and a.is_floating_point() else a for a in example_args]
            r32 = m32(*args32)
            r32 = r32 if isinstance(r32, (list, tuple)) else [r32]
        else:
            r32 = refs
    e32 = [max_rel_err(o.reshape(-1), r.float().reshape(-1)) for o, r in zip(outs, r32)]
    l2 = [rel_l2(o.reshape(-1), r.float().reshape(-1)) for o, r in zip(outs, r32)]
    d = {"max_rel_err": max(e32), "per_output": e32, "rel_l2": l2, "tolerance": tolerance, "ok": max(e32) <= tolerance,
         "oracle": "eager fp32 on the model's weights" if low else "eager model"}
    if low:
        d["vs_eager_model_dtype"] = [max_rel_err(o.reshape(-1), r.float().reshape(-1)) for o, r in zip(outs, refs)]
    return d


def measure(res: CompileResult, example_args, iters: int) -> dict[str, Any]:
    """Device time of the forward (CUDA events over ``iters`` forwards) and of
    every launch on its own (events around each launch, a short device sleep
    ahead of it so host launch cost stays out), the numbers the cost report
    sets against the model."""
    mod = res.module
    dev_args = [a.to(res.config.device) for a in example_args]
    for _ in range(3):
        mod(*dev_args)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        mod(*dev_args)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / iters
    per_launch: dict[str, list[float]] = {}
    mk = lambda: torch.cuda.Event(enable_timing=True)
    with torch.cuda.device(mod.device):
        stream = torch.cuda.current_stream()
        for _ in range(max(1, min(iters, 10))):
            marks = []
            for launch in mod.launches:
                torch.cuda._sleep(100_000)
                a, b = mk(), mk()
                a.record(stream)
                launch.fn()
                b.record(stream)
                marks.append((launch.name, a, b))
            torch.cuda.synchronize()
            for name, a, b in marks:
                per_launch.setdefault(name, []).append(a.elapsed_time(b) * 1e3)
    kernel_us = {k: sorted(v)[len(v) // 2] for k, v in per_launch.items()}
    tokens = res.program.tensors[res.program.inputs[0]].shape[0]
    return {"ms_per_forward": ms, "tokens": tokens, "tokens_per_s": tokens / (ms / 1e3), "iters": iters,
            "kernels": mod.n_launches, "cuda_graph": mod._graph is not None, "kernel_us": kernel_us}


# ---------------------------------------------------------------- reports
def plan_report(result: PlanResult, hw: B200Spec, config: CompileConfig) -> str:
    lines = [f"# Partition plan ({config.run_name})", "",
             f"Hardware: {hw.name} ({hw.source} peaks): {hw.sm_count} SMs, HBM {hw.hbm_gbs:,.0f} GB/s, "
             f"bf16 {hw.bf16_tflops:,.0f} TFLOP/s",
             f"Candidates: {len(result.candidates)} (legal: {sum(c.legal for c in result.candidates)}), planner mode: "
             f"{config.planner_mode}", "", "| # | kernels | est. us | legal | note |", "|---|---|---|---|---|"]
    for c in sorted(result.candidates, key=lambda c: (not c.legal, c.total_us)):
        note = c.error or "; ".join(c.violations[:2]) or ("best" if c is result.best else "")
        est = f"{c.total_us:,.1f}" if c.legal else "-"
        lines.append(f"| {c.index} | {len(c.program.kernels) if c.program else '-'} | {est} | {'yes' if c.legal else 'no'} | {note} |")
    lines += ["", "## Chosen program", "", "```", result.program.summary(), "```"]
    notes = check_program(result.program).notes
    if notes:  # legal kernels that run on a slower device path
        lines += ["", "## Device paths", ""] + [f"- {n}" for n in notes]
    return "\n".join(lines)


def cost_report_json(program: Program, hw: B200Spec, config: CompileConfig) -> dict[str, Any]:
    kernels = [{"name": k.name, "kind": k.kind, "tiles": k.tiles, "us": k.cost.get("us"),
                "breakdown": k.cost.get("breakdown", {})} for k in program.kernels]
    inter = program.intermediates()
    link = {t: program.tensors[t].nbytes for t in inter}
    return {"hw": hw.summary(), "kernel_launch_overhead_us": config.kernel_launch_overhead_us, "kernels": kernels,
            "total_us": program.metadata.get("plan", {}).get("total_us"), "intermediate_tensors": link,
            "intermediate_bytes": sum(link.values())}


def cost_report_md(program: Program, hw: B200Spec, config: CompileConfig, measured: dict | None = None) -> str:
    total = program.metadata.get("plan", {}).get("total_us", 0.0)
    lines = [f"# Cost report ({program.name})", "",
             f"B200 roofline model ({hw.source} peaks): estimated forward **{total:,.1f} us** incl. "
             f"{config.kernel_launch_overhead_us} us per launch.", ""]
    if measured:
        lines += [f"Measured on the device: **{measured['ms_per_forward'] * 1e3:,.1f} us** per forward "
                  f"({measured['tokens_per_s']:,.0f} tokens/s).", ""]
    timed = (measured or {}).get("kernel_us", {})
    lines += ["| kernel | kind | tiles | est. us | measured us | measured / est. | bound | flops | bytes |",
              "|---|---|---|---|---|---|---|---|---|"]
    for k in program.kernels:
        b = k.cost.get("breakdown", {})
        est = k.cost.get("us", 0.0)
        got = timed.get(k.name)
        got_s = f"{got:,.2f}" if got is not None else "-"
        ratio = f"{got / est:.2f}" if got is not None and est else "-"
        lines.append(f"| {k.name} | {k.kind} | {k.tiles} | {est:,.2f} | {got_s} | {ratio} | {b.get('bound', '-')} | "
                     f"{b.get('flops', 0):.3g} | {b.get('bytes', 0):.3g} |")
    extra = {n: v for n, v in timed.items() if n not in {k.name for k in program.kernels}}
    for n, v in extra.items():  # launches the runtime adds (row statistics, collectives)
        lines.append(f"| {n} | runtime | - | - | {v:,.2f} | - | - | - | - |")
    cal = hw.calibration
    if cal:
        lines += ["", f"Model terms fitted on {cal.get('when', '?')} to event-timed kernels of "
                      f"{', '.join(sorted(cal.get('sources', {})))} (torch_helion.cost_models.calibrate)."]
    inter = program.intermediates()
    lines += ["", f"Kernel-to-kernel links: {len(inter)} tensors, "
                  f"{sum(program.tensors[t].nbytes for t in inter):,} bytes through HBM."]
    return "\n".join(lines) + "\n"
