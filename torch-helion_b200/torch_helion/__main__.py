"""Command line: compile a model, and optionally run and time it on a B200.

::

    python -m torch_helion --config c2 --run --bench 20
    python -m torch_helion --model workloads.llama_block:build_llama_block --shape seq=512 --run
    torchrun --nproc-per-node 8 -m torch_helion --config c3 --run --bench 10 --world-size 8

The reference's entry points (src/torch_helion/__main__.py:35-71 and
cmd/generate_kernels.py:41-74) compile a ``module:factory`` model and print
the program, the reference check and the modelled cost; this one keeps
those options (``--model``, ``--shape``, ``--run-name``, ``--results-dir``,
``--hw-spec``, ``--planner``, ``--save-params``, ``--no-check``) and adds
the B200 ones:

``--backend b200``   the only backend of this package (the reference's
                     Helion/Loom emission is not built)
``--config cN``      a BASELINE configuration from ``workloads.configs``
``--run``            build the device program and run the forward on the
                     GPU (without it: compile only, artefacts on disk, no
                     GPU needed -- the ``generate_kernels`` loop)
``--bench N``        time N forwards with CUDA events (after 3 warm-ups)
``--world-size N``   tensor parallelism over N ranks (launch with torchrun;
                     one process per GPU, NCCL)

Exit status 0 when the compile succeeded and, with ``--run``, the reference
check passed.
"""

from __future__ import annotations

import argparse
import importlib
import inspect
import logging
import os
import sys
from pathlib import Path

from .config import DEFAULT_HW_SPEC, DEFAULT_RESULTS_DIR, REPO_ROOT, PKG_ROOT, CompileConfig


def _shape_overrides(items: list[str]) -> dict[str, int]:
    out = {}
    for item in items:
        key, sep, value = item.partition("=")
        if not sep:
            raise SystemExit(f"--shape expects KEY=INT, got {item!r}")
        out[key] = int(value)
    return out


def _build_model(args):
    for p in (str(PKG_ROOT), str(REPO_ROOT)):
        if p not in sys.path:
            sys.path.insert(0, p)
    overrides = _shape_overrides(args.shape)
    if args.config:
        from workloads import configs

        factory = {"c1": configs.c1_llama_fp32, "c2": configs.c2_mamba_block_bf16, "c3": configs.c3_llama8b_bf16,
                   "c4": configs.c4_mamba24_bf16}[args.config]
        cfg = factory()
        for k, v in overrides.items():
            if not hasattr(cfg, k):
                raise SystemExit(f"--shape {k}: {type(cfg).__name__} has no field {k}")
            setattr(cfg, k, v)
        return configs.build(cfg, seed=0)
    mod_name, _, fn_name = args.model.partition(":")
    module = importlib.import_module(mod_name)
    factory = getattr(module, fn_name or "build")
    if not overrides:
        return factory()
    cfg_types = [c for n, c in inspect.getmembers(module, inspect.isclass) if n.endswith("Config") and c.__module__ == module.__name__]
    if not cfg_types:
        raise SystemExit(f"--shape needs a *Config class in {mod_name}")
    return factory(cfg_types[0](**overrides))


def main(argv: list[str] | None = None) -> int:
    p = argparse.ArgumentParser(prog="torch_helion", description="Compile a PyTorch model to sm_100a kernels and run it.")
    p.add_argument("--model", default="workloads.llama_block:build_llama_block", help="module:factory building the model")
    p.add_argument("--config", choices=["c1", "c2", "c3", "c4"], help="a BASELINE configuration instead of --model")
    p.add_argument("--shape", action="append", default=[], metavar="KEY=INT", help="model config override (repeatable)")
    p.add_argument("--run-name", default=None)
    p.add_argument("--results-dir", type=Path, default=DEFAULT_RESULTS_DIR)
    p.add_argument("--hw-spec", type=Path, default=DEFAULT_HW_SPEC)
    p.add_argument("--planner", choices=["exhaustive", "greedy"], default="exhaustive")
    p.add_argument("--save-params", action="store_true")
    p.add_argument("--no-check", action="store_true", help="skip the reference check against the eager model")
    p.add_argument("--no-verify-passes", action="store_true", help="skip the per-pass numeric re-verification")
    p.add_argument("--backend", default="b200", choices=["b200"])
    p.add_argument("--device", default=None, help="CUDA device (default cuda:LOCAL_RANK)")
    p.add_argument("--run", action="store_true", help="run the forward on the GPU")
    p.add_argument("--bench", type=int, default=0, metavar="N", help="time N forwards (implies --run)")
    p.add_argument("--cuda-graph", action="store_true", help="replay the forward as one CUDA graph")
    p.add_argument("--world-size", type=int, default=1, help="tensor-parallel ranks (launch with torchrun)")
    p.add_argument("--tp-chunks", type=int, default=4)
    p.add_argument("--tp-comm-sms", type=int, default=None, help="SMs the overlapped GEMMs leave to the all-reduces")
    p.add_argument("--tp-allreduce", choices=["auto", "multimem", "nccl"], default="auto")
    p.add_argument("-v", "--verbose", action="store_true")
    args = p.parse_args(argv)
    logging.basicConfig(level=logging.INFO if args.verbose else logging.WARNING, format="%(asctime)s %(message)s")

    run = args.run or args.bench > 0
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.world_size > 1:
        if not run:
            raise SystemExit("--world-size needs --run (the shards run on the GPUs)")
        import torch
        import torch.distributed as dist
        from datetime import timedelta

        if int(os.environ.get("WORLD_SIZE", "1")) != args.world_size:
            raise SystemExit(f"--world-size {args.world_size}: launch with torchrun --nproc-per-node {args.world_size}")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    from .pipeline import compile_model

    model = _build_model(args)
    (example,) = model.example_inputs(seed=1) if "seed" in inspect.signature(model.example_inputs).parameters \
        else model.example_inputs()
    name = args.run_name or (args.config or args.model.split(":")[-1]) + (f"_r{rank}" if args.world_size > 1 else "")
    cfg = CompileConfig(run_name=name, results_dir=args.results_dir, hw_spec=args.hw_spec, planner_mode=args.planner,
                        save_params=args.save_params, backend=args.backend, device=args.device or f"cuda:{local}",
                        execute=run, verify_passes=not args.no_verify_passes,
                        reference_check=run and not args.no_check and args.world_size == 1,
                        cuda_graph=args.cuda_graph and args.world_size == 1, world_size=args.world_size,
                        tp_mode="heads" if args.world_size > 1 else None, tp_chunks=args.tp_chunks,
                        tp_comm_sms=args.tp_comm_sms, tp_allreduce=args.tp_allreduce,
                        measure_iters=args.bench)
    res = compile_model(model, (example,), cfg)
    ok = True
    if rank == 0:
        print(res.program.summary())
        print(f"modelled forward: {res.estimated_us:,.1f} us (B200 roofline model); results in {res.run_dir}")
        if res.reference_check:
            rc = res.reference_check
            ok = bool(rc["ok"])
            print(f"reference check: max rel err {rc['max_rel_err']:.3e}, rel-L2 {max(rc['rel_l2']):.3e} "
                  f"({'ok' if ok else 'FAILED'}; {rc['oracle']})")
        if res.measured:
            m = res.measured
            print(f"measured: {m['ms_per_forward'] * 1e3:,.1f} us per forward, {m['tokens_per_s']:,.0f} tokens/s "
                  f"({m['kernels']} kernels, CUDA graph {'on' if m['cuda_graph'] else 'off'}, {m['iters']} iterations)")
    if args.world_size > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    raise SystemExit(main())
