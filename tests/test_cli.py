"""``python -m torch_helion``: the reference's command-line entry
(src/torch_helion/__main__.py:35-71) with the B200 options.  Compile-only runs
need no GPU; ``--run --bench`` runs on one."""

from __future__ import annotations

import json

import pytest


def _main(argv):
    from torch_helion.__main__ import main

    return main(argv)


def test_compile_only_baseline_config(tmp_path, capsys):
    assert _main(["--config", "c1", "--results-dir", str(tmp_path), "--run-name", "c1", "--no-verify-passes"]) == 0
    out = capsys.readouterr().out
    assert "k0_gemm" in out and "modelled forward" in out
    run = tmp_path / "c1"
    for f in ("06_opir.json", "07_launch_plan.json", "09_cost_report.md", "manifest.json"):
        assert (run / f).exists(), f
    manifest = json.loads((run / "manifest.json").read_text())
    assert any(a["name"] == "06_opir.json" and a["stage"] == "plan" for a in manifest)


def test_model_factory_with_shape_overrides(tmp_path, capsys):
    argv = ["--model", "workloads.mamba:build_mamba_model", "--shape", "batch=1", "--shape", "seq=128",
            "--shape", "d_model=64", "--shape", "headdim=16", "--shape", "d_state=16", "--shape", "chunk=32",
            "--results-dir", str(tmp_path), "--run-name", "m"]
    assert _main(argv) == 0
    assert "ssd" in capsys.readouterr().out


def test_rejects_unknown_shape_field(tmp_path):
    with pytest.raises(SystemExit):
        _main(["--config", "c1", "--shape", "nonsense=3", "--results-dir", str(tmp_path)])


@pytest.mark.gpu
def test_run_and_bench_on_gpu(tmp_path, capsys):
    argv = ["--config", "c2", "--shape", "batch=1", "--shape", "seq=512", "--run", "--bench", "3",
            "--results-dir", str(tmp_path), "--run-name", "c2"]
    assert _main(argv) == 0
    out = capsys.readouterr().out
    assert "reference check" in out and "ok" in out and "measured" in out
