"""Fit the B200 cost model to event-timed kernels of this build.

::

    python -m torch_helion.cost_models.calibrate \\
        --measured c2=bench_c2.json --measured c3=bench_c3.json [--out b200_calibration.json]

Each ``--measured name=path`` pairs a BASELINE workload (``workloads.configs``)
with a file whose last line is a ``bench.py`` JSON line: its ``kernels_ms``
holds the CUDA-event time of every launch of that workload's forward.  The
workload is compiled here (CPU, no GPU needed), every kernel is costed with
the current model, and the model's free terms are refitted:

* GEMMs (tcgen05): ``t = gemm_fixed_us + waves x tile_work / e_mma``, a
  weighted least-squares fit of the fixed cost and 1/e_mma over all GEMMs
  (relative residuals, so small and large GEMMs count alike);
* attention: ``e_attn`` from ``t - fixed = flops / (peak x e_attn)``;
* SSD scans: ``e_ssd_mem`` from their bytes against the HBM peak;
* conv / norms / row statistics: a least-squares fit of the fixed cost and
  1/e_elem against their bytes.

It writes the new values with the per-kernel table (modelled before,
measured, modelled after) so the fit is auditable; the reference keeps the
same kind of analytic-vs-measured table for its Loom backend
(docs/cost_models.md:51-88).
"""

from __future__ import annotations

import argparse
import json
import math
import sys
import time
from pathlib import Path
from typing import Any

from .b200 import CALIBRATION_FILE, B200Spec, search_tiles

_FITTED = ("eff_mma", "gemm_fixed_us", "eff_attn", "attn_fixed_us", "eff_ssd_mem", "ssd_fixed_us", "eff_elem",
           "elem_fixed_us")


def _workload_program(name: str):
    from torch_helion import CompileConfig, compile_model
    from workloads import configs

    factory = {"c1": configs.c1_llama_fp32, "c2": configs.c2_mamba_block_bf16, "c3": configs.c3_llama8b_bf16,
               "c4": configs.c4_mamba24_bf16}[name]
    cfg = factory()
    model = configs.build(cfg, seed=0)
    (x,) = model.example_inputs(seed=1)
    import tempfile

    with tempfile.TemporaryDirectory() as d:
        res = compile_model(model, (x,), CompileConfig(run_name=name, results_dir=d, execute=False, verify_passes=False))
    return res.program


def _linfit(xs: list[float], ts: list[float]) -> tuple[float, float]:
    """(f, u) minimising sum(((f + u x_i - t_i) / t_i)^2), f >= 0."""
    w = [1.0 / (t * t) for t in ts]
    s0 = sum(w)
    sx = sum(wi * x for wi, x in zip(w, xs))
    sxx = sum(wi * x * x for wi, x in zip(w, xs))
    st = sum(wi * t for wi, t in zip(w, ts))
    sxt = sum(wi * x * t for wi, x, t in zip(w, xs, ts))
    det = s0 * sxx - sx * sx
    if len(xs) >= 2 and abs(det) > 1e-30:
        f = (sxx * st - sx * sxt) / det
        u = (s0 * sxt - sx * st) / det
        if f >= 0 and u > 0:
            return f, u
    return 0.0, sxt / sxx if sxx > 0 else 1.0  # through the origin


def fit(records: list[dict[str, Any]], hw: B200Spec) -> dict[str, float]:
    """New values of the fitted terms from per-kernel records (see module doc)."""
    out: dict[str, float] = {}
    gemms = [r for r in records if r["kind"] == "gemm" and r["dtype"] != "float32"]
    if gemms:
        xs = [r["waves"] * 128 * r["tile_n"] * r["K"] * 2 / (hw.sm_tflops * 1e12) * 1e6 for r in gemms]
        f, u = _linfit(xs, [r["measured_us"] for r in gemms])
        out["gemm_fixed_us"], out["eff_mma"] = f, min(1.2, 1.0 / u)
    fixed = out.get("gemm_fixed_us", hw.gemm_fixed_us)
    att = [r for r in records if r["kind"] == "attention" and r["dtype"] != "float32"]
    if att:
        effs = [r["flops"] / (hw.bf16_tflops * 1e12) * 1e6 / max(r["measured_us"] - fixed, 1e-3) for r in att]
        out["eff_attn"], out["attn_fixed_us"] = sum(effs) / len(effs), fixed
    ssd = [r for r in records if r["kind"] == "ssd"]
    if ssd:
        effs = [r["bytes"] / (hw.hbm_gbs * 1e9) * 1e6 / max(r["measured_us"] - fixed, 1e-3) for r in ssd]
        out["eff_ssd_mem"], out["ssd_fixed_us"] = sum(effs) / len(effs), fixed
    elem = [r for r in records if r["kind"] not in ("gemm", "attention", "ssd")]
    if elem:
        xs = [r["bytes"] / (hw.hbm_gbs * 1e9) * 1e6 for r in elem]
        f, u = _linfit(xs, [r["measured_us"] for r in elem])
        out["elem_fixed_us"], out["eff_elem"] = f, min(1.2, 1.0 / u)
    return out


def records_for(name: str, kernels_ms: dict[str, float], hw: B200Spec) -> list[dict[str, Any]]:
    """One record per kernel of workload ``name`` that has a measured time."""
    prog = _workload_program(name)
    recs = []
    for spec in prog.kernels:
        if spec.name not in kernels_ms:
            continue
        best = search_tiles(spec, prog.tensors, hw).best
        dtype = prog.tensors[spec.args[0].tensor].dtype
        recs.append(dict(workload=name, kernel=spec.name, kind=spec.kind, dtype=dtype, measured_us=kernels_ms[spec.name] * 1e3,
                         modelled_us=best.us, flops=best.flops, bytes=best.bytes, tile_n=best.tiles.get("tile_n", 0),
                         waves=best.details.get("waves", 0), K=spec.k_extent))
    return recs


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(prog="torch_helion.cost_models.calibrate")
    ap.add_argument("--measured", action="append", required=True, metavar="WORKLOAD=PATH",
                    help="a BASELINE workload (c1..c4) and a bench.py JSON line with its kernels_ms")
    ap.add_argument("--out", type=Path, default=CALIBRATION_FILE)
    args = ap.parse_args(argv)
    root = Path(__file__).resolve().parents[3]
    for p in (str(root / "torch-helion_b200"), str(root)):
        if p not in sys.path:
            sys.path.insert(0, p)
    hw = B200Spec.load()
    records: list[dict[str, Any]] = []
    sources = {}
    for item in args.measured:
        name, _, path = item.partition("=")
        line = json.loads(Path(path).read_text().strip().splitlines()[-1])
        records += records_for(name, line["kernels_ms"], hw)
        sources[name] = {"file": Path(path).name, "clocks": line.get("clocks"), "workload": line["config"]["workload"]}
    values = fit(records, hw)
    after = B200Spec.load().apply_calibration({"values": values})
    prog_cache: dict[str, Any] = {}
    for r in records:
        prog = prog_cache.setdefault(r["workload"], _workload_program(r["workload"]))
        spec = next(k for k in prog.kernels if k.name == r["kernel"])
        r["modelled_after_us"] = search_tiles(spec, prog.tensors, after).best.us
    cal = {"values": values, "fitted": list(_FITTED), "sources": sources,
           "when": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()),
           "peaks": {"hbm_gbs": hw.hbm_gbs, "bf16_tflops": hw.bf16_tflops, "source": hw.source},
           "kernels": [{k: (round(v, 3) if isinstance(v, float) else v) for k, v in r.items()
                        if k in ("workload", "kernel", "kind", "measured_us", "modelled_us", "modelled_after_us")}
                       for r in records]}
    args.out.write_text(json.dumps(cal, indent=1) + "\n")
    print(f"{'workload':8s} {'kernel':18s} {'kind':14s} {'before':>10s} {'measured':>10s} {'after':>10s}")
    for r in records:
        print(f"{r['workload']:8s} {r['kernel']:18s} {r['kind']:14s} {r['modelled_us']:10.1f} {r['measured_us']:10.1f} "
              f"{r['modelled_after_us']:10.1f}")
    print(json.dumps(values, indent=1))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
