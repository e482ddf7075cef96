"""Workloads: the models torch-helion is benchmarked on, plus the BASELINE
configurations (C1-C5) with their seeded synthetic inputs.

``TARGETS`` mirrors the reference's registry (models/__init__.py:14-49) so
``load_model("mamba")``-style entry points keep working.
"""

from __future__ import annotations

import importlib
from typing import Any

TARGETS: dict[str, tuple[str, str, str]] = {
    "llama_block": ("workloads.llama_block", "build_llama_block",
                    "one Llama-style decoder block: RMSNorm, QKV + RoPE, attention, SwiGLU MLP"),
    "mamba": ("workloads.mamba", "build_mamba_model", "a Mamba-2 backbone: stacked SSD blocks with a final norm"),
    "mamba_block": ("workloads.mamba", "build_mamba_block", "a single Mamba-2 block"),
}


def available() -> list[str]:
    return list(TARGETS)


def resolve(name: str) -> tuple[Any, str]:
    if name not in TARGETS:
        raise KeyError(name)
    mod, factory, _ = TARGETS[name]
    return getattr(importlib.import_module(mod), factory), f"{mod}:{factory}"
