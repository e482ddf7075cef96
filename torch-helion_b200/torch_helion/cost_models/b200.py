"""B200 cost model: the reference's analytic model retargeted to sm_100a.

The reference estimates Loom cycles per kernel from per-tile load/compute
terms on an 8x8 mesh (src/torch_helion/cost_models/analytic.py:109-256)
and searches 32-aligned tiles that fit L1 (tile_search.py:56-71).  Here a
kernel's time is a calibrated roofline of the kernel this build launches
for it:

* GEMM (tcgen05):  fixed + waves x (128 x BN x K MMA work / (SM peak x e_mma)),
                   tiles = ceil(T/128) x ceil(N/BN) over the SMs, BN searched
                   in {128, 256}; never below the HBM time of its bytes;
* GEMM (fp32):     the same over FFMA tiles of 32 x 128 (e_simt);
* attention:       fixed + flops / (bf16 peak x e_attn) (half the flops when causal);
* SSD scan:        fixed + max(flops / (bf16 peak x e_ssd_tc), bytes / (HBM x e_ssd_mem));
* conv / norms / row statistics / embedding: fixed + bytes / (HBM x e_elem).

The peaks come from ``MEASURED_PEAKS.json`` (driver-measured on this pool;
nominal B200 figures otherwise) and the efficiencies and fixed costs from
``b200_calibration.json`` beside this file, fitted to event-timed kernels
of this build by :mod:`torch_helion.cost_models.calibrate`.
"""

from __future__ import annotations

import json
import math
import os
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any

from ..capture.opgraph import TensorType
from ..optimizer.opir import KernelSpec

DTYPE_BYTES = {"float32": 4, "bfloat16": 2, "float16": 2, "int64": 8}


class CostModelError(ValueError):
    pass


@dataclass
class B200Spec:
    name: str = "B200"
    sm_count: int = 148
    hbm_gbs: float = 8000.0          # GB/s (nominal HGX 7.7-8 TB/s)
    bf16_tflops: float = 2250.0      # dense tensor peak
    fp32_tflops: float = 72.0        # FFMA: 148 SMs x 128 lanes x 2 x ~1.9 GHz
    smem_per_cta: int = 227 * 1024
    tmem_cols: int = 512
    l2_bytes: int = 126 * 1024 * 1024
    launch_us: float = 3.0
    source: str = "nominal"
    path: Path | None = None

    # efficiencies of this build's kernels against the peaks and fixed costs
    # per launch (us), fitted to measured kernel times (b200_calibration.json)
    eff_mma: float = 0.8
    gemm_fixed_us: float = 5.0
    eff_simt: float = 0.35
    eff_attn: float = 0.35
    attn_fixed_us: float = 5.0
    eff_ssd_tc: float = 0.2
    eff_ssd_mem: float = 0.2
    ssd_fixed_us: float = 5.0
    eff_elem: float = 0.6
    elem_fixed_us: float = 5.0
    calibration: dict[str, Any] = field(default_factory=dict)
    tile_widths: tuple[int, ...] = (128, 256)

    @staticmethod
    def load(path: str | Path | None = None) -> "B200Spec":
        cands = [Path(path)] if path else []
        env = os.environ.get("TORCH_HELION_B200_PEAKS")
        if env:
            cands.append(Path(env))
        cands.append(Path(__file__).resolve().parents[3] / "MEASURED_PEAKS.json")
        spec = B200Spec()
        for p in cands:
            if p and p.is_file() and p.suffix == ".json":
                d = json.loads(p.read_text())
                spec = B200Spec(hbm_gbs=float(d.get("hbm_gbs", 8000.0)), bf16_tflops=float(d.get("bf16_tflops", 2250.0)),
                                source="measured", path=p)
                break
        spec.apply_calibration(load_calibration())
        return spec

    def apply_calibration(self, cal: dict[str, Any] | None) -> "B200Spec":
        """Take the fitted efficiencies / fixed costs of a calibration record."""
        if cal:
            for k, v in cal.get("values", {}).items():
                if hasattr(self, k):
                    setattr(self, k, float(v))
            self.calibration = {k: v for k, v in cal.items() if k != "values"}
        return self

    @property
    def sm_tflops(self) -> float:
        return self.bf16_tflops / self.sm_count

    @property
    def ridge(self) -> float:
        return self.bf16_tflops * 1e12 / (self.hbm_gbs * 1e9)

    def summary(self) -> dict[str, Any]:  # noqa: D401 - artefact 04_hw_spec.json
        d = asdict(self)
        d["path"] = str(self.path) if self.path else None
        d["ridge_flop_per_byte"] = self.ridge
        return d


@dataclass
class CostBreakdown:
    us: float
    tiles: dict[str, int]
    flops: float
    bytes: float
    t_compute_us: float
    t_memory_us: float
    bound: str
    details: dict[str, Any] = field(default_factory=dict)

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


def _eb(t: TensorType) -> int:
    return DTYPE_BYTES.get(t.dtype, 4)


def _arg_bytes(spec: KernelSpec, tensors: dict[str, TensorType], roles: tuple[str, ...] | None = None) -> float:
    tot = 0.0
    for a in spec.args:
        if roles is not None and a.role not in roles:
            continue
        t = tensors[a.tensor]
        w = (a.cols[1] - a.cols[0]) if a.cols else (t.shape[-1] if t.rank else 1)
        rows = t.shape[0] if t.rank == 2 else 1
        tot += rows * w * _eb(t)
    return tot


def gemm_cost(spec: KernelSpec, tensors: dict[str, TensorType], hw: B200Spec, bn: int) -> CostBreakdown:
    T, N, K = spec.grid["rows"], spec.grid["cols"], spec.k_extent
    dt = tensors[spec.args[0].tensor].dtype
    eb = DTYPE_BYTES.get(dt, 2)
    flops = 2.0 * T * N * K
    out_bytes = sum(tensors[o.tensor].numel * eb for o in spec.outputs)
    byts = T * K * eb + N * K * eb + out_bytes + _arg_bytes(spec, tensors, ("extra",))
    if dt == "float32":
        # 32x128 FFMA tiles, several resident per SM
        tiles = math.ceil(T / 32) * math.ceil(N / 128)
        waves = math.ceil(tiles / hw.sm_count)
        per_tile = 32 * 128 * K * 2 / (hw.fp32_tflops * 1e12 / hw.sm_count * hw.eff_simt)
        t_c = waves * per_tile * 1e6 + hw.gemm_fixed_us
    else:
        if bn not in hw.tile_widths:
            raise CostModelError(f"tile width {bn} not built")
        # the last column tile multiplies only its live width (rounded to 16)
        tiles = math.ceil(T / 128) * math.ceil(N / bn)
        n_eff = (N // bn) * bn + (math.ceil((N % bn) / 16) * 16 if N % bn else 0)
        waves = math.ceil(math.ceil(T / 128) * n_eff / bn / hw.sm_count)
        per_tile = 128 * bn * K * 2 / (hw.sm_tflops * 1e12 * hw.eff_mma)
        t_c = waves * per_tile * 1e6 + hw.gemm_fixed_us
    t_m = byts / (hw.hbm_gbs * 1e9) * 1e6
    us = max(t_c, t_m)
    return CostBreakdown(us, {"tile_m": 128 if dt != "float32" else 32, "tile_n": bn, "tile_k": 64}, flops, byts, t_c,
                         t_m, "tensor" if t_c >= t_m else "hbm", {"tiles": tiles, "waves": waves})


def macro_cost(spec: KernelSpec, tensors: dict[str, TensorType], hw: B200Spec) -> CostBreakdown:
    a = spec.attrs
    out = tensors[spec.outputs[0].tensor]
    eb = _eb(out)
    byts = _arg_bytes(spec, tensors) + out.numel * eb
    flops, t_c, t_m = 0.0, 0.0, 0.0
    peak = hw.bf16_tflops * 1e12
    if spec.kind == "attention":
        b, s, h, d = a["batch"], a["seq"], a["heads"], a["head_dim"]
        flops = 4.0 * b * h * s * s * d * (0.5 if a.get("causal") else 1.0)
        if eb == 4:  # fp32 models run the SIMT flash kernel
            t_c = flops / (hw.fp32_tflops * 1e12 * hw.eff_simt) * 1e6 + hw.attn_fixed_us
        else:
            t_c = flops / (peak * hw.eff_attn) * 1e6 + hw.attn_fixed_us
        t_m = byts / (hw.hbm_gbs * 1e9) * 1e6
    elif spec.kind == "ssd":
        b, s, h, p, n = a["batch"], a["seq"], a["heads"], a["head_dim"], a["state_dim"]
        L = min(256, s)
        flops = b * s * h * (2 * L * p + 4 * p * n + 2 * L * n / max(1, h // a["ngroups"]))
        byts += 2 * b * math.ceil(s / L) * h * p * n * 2  # chunk states (2-byte), written and read
        t_c = flops / (peak * hw.eff_ssd_tc) * 1e6 + hw.ssd_fixed_us
        t_m = byts / (hw.hbm_gbs * 1e9 * hw.eff_ssd_mem) * 1e6 + hw.ssd_fixed_us
    else:
        t_m = byts / (hw.hbm_gbs * 1e9 * hw.eff_elem) * 1e6 + hw.elem_fixed_us
    return CostBreakdown(max(t_c, t_m), {}, flops, byts, t_c, t_m, "compute" if t_c >= t_m else "hbm")


@dataclass
class TileSearchResult:
    best: CostBreakdown
    evaluated: int
    feasible: int
    top: list[CostBreakdown]


def search_tiles(spec: KernelSpec, tensors: dict[str, TensorType], hw: B200Spec) -> TileSearchResult:
    """Cheapest tile width for a GEMM (other kinds have fixed tiles)."""
    if spec.kind != "gemm":
        c = macro_cost(spec, tensors, hw)
        return TileSearchResult(c, 1, 1, [c])
    res = []
    for bn in hw.tile_widths:
        if bn == 256 and spec.grid["cols"] < 256:
            continue
        res.append(gemm_cost(spec, tensors, hw, bn))
    res.sort(key=lambda r: r.us)
    return TileSearchResult(res[0], 2, len(res), res)


def kernel_cost(spec: KernelSpec, tensors: dict[str, TensorType], hw: B200Spec) -> CostBreakdown:
    return search_tiles(spec, tensors, hw).best


CALIBRATION_FILE = Path(__file__).with_name("b200_calibration.json")


def load_calibration(path: str | Path | None = None) -> dict[str, Any] | None:
    """The committed fit (or the file ``$TORCH_HELION_B200_CALIBRATION`` / ``path`` names)."""
    p = Path(path or os.environ.get("TORCH_HELION_B200_CALIBRATION", CALIBRATION_FILE))
    return json.loads(p.read_text()) if p.is_file() else None
