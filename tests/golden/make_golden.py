"""Generate the golden fixtures under tests/golden/ from the REFERENCE code.

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py [--ref /path/to/torch-helion]

The reference checkout (--ref, or $TH_REFERENCE; required) is only
needed here, when the fixtures are (re)generated; the tests read the
committed ``*.pt`` files and never import the reference.  Every fixture is
produced by the reference's own modules (models/llama_block.py,
models/mamba.py) with their own seeded builders, so the oracle and the
workload builders are pinned to the reference's behaviour:

* ``llama_small_fp32.pt``   full state dict + input + eager output (small block)
* ``mamba_small_chunked.pt``  2-layer backbone, chunked scan, conv, ngroups=1
* ``mamba_small_quadratic.pt`` reference defaults (quadratic, per-head groups, no conv)
* ``ssd_known_answer.pt``   reference ssd_chunked / ssd_quadratic on the
                            reference test inputs (tests/test_mamba.py:41-66)
* ``c1_llama.pt``           C1 shape: weight samples, input, eager output
* ``c2_mamba.pt``           C2 shape: weight samples + output statistics of
                            the fp32 eager forward on bf16 weights/inputs
"""

from __future__ import annotations

import argparse
import math
import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def _samples(sd: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """First 16 values and fp64 sum/abs-sum of every parameter."""
    out = {}
    for k, v in sd.items():
        f = v.detach().double().reshape(-1)
        out[k] = torch.cat((f[:16], torch.tensor([f.sum().item(), f.abs().sum().item()], dtype=torch.float64)))
    return out


def _baseline_a(model, seed: int = 0) -> None:
    """BASELINE A distribution A = -exp(U[log 1, log 16]) (same draw as
    workloads.mamba.apply_baseline_init)."""
    gen = torch.Generator().manual_seed(10_000 + seed)
    with torch.no_grad():
        for name, prm in model.named_parameters():
            if name.endswith("A_log"):
                prm.copy_((torch.rand(prm.shape, generator=gen) * math.log(16.0)).to(prm.dtype))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("TH_REFERENCE"),
                    help="checkout of the reference project (or set $TH_REFERENCE)")
    a = ap.parse_args()
    if not a.ref:
        ap.error("give the reference checkout with --ref or $TH_REFERENCE")
    sys.path.insert(0, a.ref)
    from models.llama_block import LlamaBlockConfig, build_llama_block
    from models.mamba import MambaConfig, build_mamba_model, causal_chunk_masks, ssd_chunked, ssd_quadratic

    # ---- small Llama block, fp32
    cfg = LlamaBlockConfig(batch=2, seq=32, hidden=64, heads=2, intermediate=128, eps=1e-6, dtype=torch.float32)
    blk = build_llama_block(cfg, seed=0)
    torch.manual_seed(1)
    x = blk.example_inputs()[0]
    with torch.no_grad():
        y = blk(x)
    torch.save({"config": dict(batch=2, seq=32, hidden=64, heads=2, intermediate=128, eps=1e-6),
                "state_dict": {k: v.clone() for k, v in blk.state_dict().items()}, "x": x, "y": y},
               HERE / "llama_small_fp32.pt")

    # ---- small Mamba backbones, fp32
    for name, kw in (
        ("mamba_small_chunked", dict(batch=2, seq=64, d_model=64, expand=2, headdim=16, d_state=16, chunk=16,
                                     n_layers=2, mode="chunked", ngroups=1, use_conv=True, dtype=torch.float32)),
        ("mamba_small_quadratic", dict(batch=2, seq=64, d_model=64, expand=2, headdim=16, d_state=16, chunk=16,
                                       n_layers=1, mode="quadratic", dtype=torch.float32)),
    ):
        mcfg = MambaConfig(**kw)
        model = build_mamba_model(mcfg, seed=0)
        if kw["mode"] == "chunked":
            _baseline_a(model)
        torch.manual_seed(1)
        u = model.example_inputs()[0]
        with torch.no_grad():
            yy = model(u)
        cfgd = {k: v for k, v in kw.items() if k != "dtype"}
        torch.save({"config": cfgd, "baseline_a": kw["mode"] == "chunked",
                    "state_dict": {k: v.clone() for k, v in model.state_dict().items() if "mask" not in k},
                    "u": u, "y": yy}, HERE / f"{name}.pt")

    # ---- SSD known answer (reference test inputs, tests/test_mamba.py:41-49)
    torch.manual_seed(0)
    b, h, s, p, n = 2, 3, 24, 4, 5
    xs = torch.randn(b, h, s, p)
    Bs = torch.randn(b, h, s, n)
    Cs = torch.randn(b, h, s, n)
    dt = torch.rand(b, h, s) * 0.1 + 0.01
    A = -(torch.rand(b, h, 1) * 0.9 + 0.1)
    dA = dt * A
    idx = torch.arange(s)
    causal = (idx.unsqueeze(1) >= idx.unsqueeze(0)).float()
    yq = ssd_quadratic(xs, dA, dt, Bs, Cs, causal)
    l, c = 6, 4
    within, across, prefix = causal_chunk_masks(l, c, torch.float32)
    r4 = lambda t: t.reshape(*t.shape[:2], c, l, t.shape[-1])
    r3 = lambda t: t.reshape(*t.shape[:2], c, l)
    yc = ssd_chunked(r4(xs), r3(dA), r3(dt), r4(Bs), r4(Cs), within, across, prefix).reshape(b, h, s, p)
    torch.save({"x": xs, "dA": dA, "dt": dt, "B": Bs, "C": Cs, "chunk": l, "y_quadratic": yq, "y_chunked": yc},
               HERE / "ssd_known_answer.pt")

    # ---- C1 shape (the reference block: multi-head, non-causal)
    cfg1 = LlamaBlockConfig(batch=1, seq=128, hidden=512, heads=8, intermediate=1408, eps=1e-6, rope_theta=10000.0,
                            dtype=torch.float32)
    blk1 = build_llama_block(cfg1, seed=0)
    torch.manual_seed(1)
    x1 = blk1.example_inputs()[0]
    with torch.no_grad():
        y1 = blk1(x1)
    torch.save({"weights": _samples(blk1.state_dict()), "x": x1, "y": y1}, HERE / "c1_llama.pt")

    # ---- C2 shape: bf16 weights, fp32 eager forward on bf16-rounded operands
    cfg2 = MambaConfig(batch=4, seq=2048, d_model=768, expand=2, headdim=64, d_state=128, chunk=256, n_layers=1,
                       mode="chunked", ngroups=1, d_conv=4, use_conv=True, dtype=torch.bfloat16)
    m2 = build_mamba_model(cfg2, seed=0)
    _baseline_a(m2)
    torch.manual_seed(1)
    u2 = m2.example_inputs()[0]
    with torch.no_grad():
        y_bf16 = m2(u2).float()
        y_f32 = m2.float()(u2.float())
    sel = (slice(None), slice(None, None, 97), slice(None, None, 13))
    torch.save({"weights": _samples({k: v for k, v in m2.state_dict().items() if "mask" not in k}),
                "u_stats": torch.tensor([u2.double().sum().item(), u2.double().abs().sum().item()], dtype=torch.float64),
                "y_sel": y_f32[sel].clone(), "y_stats": torch.tensor([y_f32.double().sum().item(),
                                                                       y_f32.double().abs().sum().item(),
                                                                       y_f32.double().pow(2).sum().item()], dtype=torch.float64),
                "eager_bf16_rel_l2": float((y_bf16 - y_f32).norm() / y_f32.norm())},
               HERE / "c2_mamba.pt")
    for f in sorted(HERE.glob("*.pt")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
