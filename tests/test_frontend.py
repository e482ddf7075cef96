"""Front end on the CPU (no GPU): capture -> canonicalisation -> partition ->
plan -> OpIR, checked the way the reference checks its optimizer
(tests/test_llama_fusion.py, tests/test_mamba_block.py: structure of the
partition, numerics of the canonical graph and of the interpreted program
against the eager model).  The programs are interpreted in fp64 by
``oracle.interpret`` and compared with the eager oracle."""

from __future__ import annotations

import json

import pytest
import torch

from conftest import rel_l2
from oracle import interpret as I
from oracle import models as O


def _compile(model, args, tmp_path, **kw):
    from torch_helion import CompileConfig, compile_model

    return compile_model(model, args, CompileConfig(run_name="fe", results_dir=tmp_path, execute=False, **kw))


def _llama(**kw):
    from workloads.llama_block import LlamaBlockConfig, build_llama_block

    base = dict(batch=2, seq=32, hidden=128, heads=4, intermediate=256, dtype=torch.float32)
    cfg = LlamaBlockConfig(**{**base, **kw})
    m = build_llama_block(cfg, 0)
    return cfg, m, m.example_inputs(seed=1)


def _mamba(**kw):
    from workloads.mamba import MambaConfig, apply_baseline_init, build_mamba_model

    base = dict(batch=2, seq=128, d_model=64, expand=2, headdim=16, d_state=16, chunk=64, n_layers=1, mode="chunked",
                ngroups=1, d_conv=4, use_conv=True, dtype=torch.float32)
    cfg = MambaConfig(**{**base, **kw})
    m = apply_baseline_init(build_mamba_model(cfg, 0), 0)
    return cfg, m, m.example_inputs(1)


def _sd(m):
    return {k: v.detach() for k, v in m.state_dict().items()}


def _mamba_ref(m, u, cfg):
    return O.mamba_forward(_sd(m), u, n_layers=cfg.n_layers, d_model=cfg.d_model, expand=cfg.expand,
                           headdim=cfg.headdim, d_state=cfg.d_state, ngroups=cfg.ngroups, chunk=cfg.chunk, eps=cfg.eps,
                           use_conv=cfg.use_conv, d_conv=cfg.d_conv, mode=cfg.mode, embedding=cfg.vocab is not None,
                           lm_head=cfg.tie_lm_head, dtype=torch.float64)


# ------------------------------------------------------------------ Llama
@pytest.mark.parametrize("kw", [dict(), dict(kv_heads=2, causal=True), dict(kv_heads=1, causal=True)],
                         ids=["mha", "gqa_causal", "mqa_causal"])
def test_llama_partition(tmp_path, kw):
    cfg, m, args = _llama(**kw)
    res = _compile(m, args, tmp_path)
    p = res.program
    assert [k.kind for k in p.kernels] == ["gemm", "attention", "gemm", "gemm", "gemm"]
    qkv, att, o, mlp, down = p.kernels
    assert len(qkv.gemms) == 3 and qkv.sumsq  # q|k|v share the normalised LHS; RMSNorm folded
    assert any(op.op == "rope" for op in qkv.epilogue)
    assert att.attrs["heads"] == cfg.heads and att.attrs["kv_heads"] == (cfg.kv_heads or cfg.heads)
    assert att.attrs["causal"] == cfg.causal and att.attrs["head_dim"] == cfg.hidden // cfg.heads
    assert len(mlp.gemms) == 2 and mlp.sumsq  # gate|up with SwiGLU epilogue
    assert {op.op for op in mlp.epilogue} >= {"silu", "mul"}
    assert any(a.role == "extra" for a in o.args) and any(a.role == "extra" for a in down.args)  # residuals
    # numerics: the interpreted program vs the eager oracle
    (x,) = args
    out = I.program_outputs(p, res.graph.params, [x])[0].reshape(x.shape)
    ref = O.llama_block_forward(_sd(m), x, heads=cfg.heads, kv_heads=cfg.kv_heads, eps=cfg.eps,
                                rope_theta=cfg.rope_theta, causal=cfg.causal, dtype=torch.float64)
    assert rel_l2(out, ref) < 1e-8  # fp32-rounded constants (RoPE tables, scale) in the graph


def test_pass_log_is_verified(tmp_path):
    _, m, args = _llama(kv_heads=2, causal=True)
    res = _compile(m, args, tmp_path)
    log = json.loads((res.run_dir / "03_pass_log.json").read_text())
    applied = [e for e in log if e.get("rewrites", 0) > 0]
    assert {e["pass"] for e in applied} >= {"match_rope", "match_rmsnorm", "match_attention"}
    for e in applied:
        assert e.get("max_rel_err", 0.0) < 1e-5, e


def test_artifacts_and_opir_roundtrip(tmp_path):
    from torch_helion.optimizer.opir import Program

    _, m, args = _llama()
    res = _compile(m, args, tmp_path)
    for f in ("01_fx_graph.txt", "02_opgraph_raw.json", "03_opgraph_canonical.json", "05_plan/plan.md", "06_opir.json",
              "07_launch_plan.json", "09_cost_report.md", "timings.json"):
        assert (res.run_dir / f).exists(), f
    loaded = Program.from_json(res.run_dir / "06_opir.json")
    assert json.dumps(loaded.to_dict(), sort_keys=True, default=str) == \
        json.dumps(json.loads(json.dumps(res.program.to_dict(), default=str)), sort_keys=True, default=str)
    assert len(res.kernel_files) == len(res.program.kernels)
    for path in res.kernel_files.values():
        plan = json.loads(path.read_text())
        assert plan["entry_point"].startswith("th_")


def test_planner_exhaustive_llama(tmp_path):
    _, m, args = _llama()
    res = _compile(m, args, tmp_path)
    meta = res.program.metadata["plan"]
    # sibling sets {q,k,v} (Bell(3)=5 partitions) and {gate,up} (Bell(2)=2)
    assert meta["search"] == "exhaustive" and meta["candidates"] == 10
    best = res.plan.best
    assert best.total_us == min(c.total_us for c in res.plan.candidates if c.legal)


def test_planner_descent_deep_mamba(tmp_path):
    cfg, m, args = _mamba(n_layers=4, use_conv=False, ngroups=8, chunk=32, seq=64, vocab=100)
    res = _compile(m, args, tmp_path)
    meta = res.program.metadata["plan"]
    assert meta["search"] == "coordinate descent" and meta["search_space"] > 512
    kinds = [k.kind for k in res.program.kernels]
    assert kinds[0] == "embedding" and kinds[-1] == "rmsnorm"
    assert kinds.count("ssd") == 4 and kinds.count("gemm") == 8  # in_proj merged, out_proj per layer
    (u,) = args
    out = I.program_outputs(res.program, res.graph.params, [u])[0]
    ref = _mamba_ref(m, u, cfg)
    assert rel_l2(out.reshape(ref.shape), ref) < 1e-6  # fp32-rounded constants (A, dt_bias folds)


# ------------------------------------------------------------------ Mamba
@pytest.mark.parametrize("kw", [dict(), dict(ngroups=None), dict(mode="quadratic", seq=64)],
                         ids=["conv_g1", "conv_per_head_groups", "quadratic"])
def test_mamba_partition(tmp_path, kw):
    cfg, m, args = _mamba(**kw)
    res = _compile(m, args, tmp_path)
    p = res.program
    assert [k.kind for k in p.kernels] == ["gemm", "causal_conv1d", "ssd", "gemm", "rmsnorm"]
    inp, conv, ssd, outp, norm_f = p.kernels
    assert conv.attrs.get("act") == "silu"
    assert ssd.attrs["gate"] and ssd.attrs["has_D"] and ssd.attrs["ngroups"] == cfg.groups
    assert ssd.attrs["heads"] == cfg.d_model * cfg.expand // cfg.headdim
    assert {a.role for a in ssd.args} == {"x", "dt", "A", "B", "C", "D", "z"}
    (u,) = args
    out = I.program_outputs(p, res.graph.params, [u])[0]
    ref = _mamba_ref(m, u, cfg)
    assert rel_l2(out.reshape(ref.shape), ref) < 1e-6  # fp32-rounded constants (A, dt_bias folds)


def test_legality_rejects_unbuilt_head_dim(tmp_path):
    from torch_helion.optimizer.legality import check_program

    _, m, args = _llama()
    res = _compile(m, args, tmp_path)
    prog = res.program
    att = next(k for k in prog.kernels if k.kind == "attention")
    att.attrs["head_dim"] = 48
    rep = check_program(prog)
    assert not rep.ok and "head_dim" in str(rep)


def _mutate(prog, kind, rule):
    """One structural fault of the named rule planted in a copy of a legal program."""
    import copy

    from torch_helion.capture.opgraph import TensorType

    prog = copy.deepcopy(prog)
    spec = next(k for k in prog.kernels if k.kind == kind)
    T = prog.tensors
    if rule == "operands":
        spec.args[0].tensor = "no_such_tensor"
    elif rule == "gemm-shape":
        spec.k_extent += 8
    elif rule == "dtype":
        rhs = next(a for a in spec.args if a.role == "rhs")
        t = T[rhs.tensor]
        T[rhs.tensor] = TensorType(t.shape, "float16" if t.dtype != "float16" else "bfloat16")
    elif rule == "attention":
        spec.attrs["kv_heads"] = 3
    elif rule == "ssd":
        spec.attrs["ngroups"] = 3
    elif rule == "conv":
        w = next(a for a in spec.args if a.role == "w")
        t = T[w.tensor]
        T[w.tensor] = TensorType((t.shape[0] + 8, t.shape[1]), t.dtype)
    elif rule == "lowering":
        spec.attrs["width"] = 7
    return prog


@pytest.mark.parametrize("model,kind,rule", [("llama", "gemm", "operands"), ("llama", "gemm", "gemm-shape"),
                                             ("llama", "gemm", "dtype"), ("llama", "attention", "attention"),
                                             ("mamba", "ssd", "ssd"), ("mamba", "causal_conv1d", "conv"),
                                             ("mamba", "causal_conv1d", "lowering")])
def test_legality_rules_name_the_broken_rule(tmp_path, model, kind, rule):
    """Every structural rule of the B200 legality check fires on a planted
    fault and names itself; the unmodified program is legal."""
    from torch_helion.optimizer.legality import check_program

    _, m, args = (_llama if model == "llama" else _mamba)(dtype=torch.bfloat16)
    prog = _compile(m, args, tmp_path).program
    assert check_program(prog).ok
    rep = check_program(_mutate(prog, kind, rule))
    assert not rep.ok
    assert rule in {v.rule for v in rep.violations}, str(rep)


def test_legality_notes_name_the_device_path(tmp_path):
    """Legal kernels on slower device paths are listed as notes (fp32 GEMMs
    on the SIMT kernel, head_dim 32 attention on the SIMT flash kernel, a
    chunk-64 scan on the three-pass path) and in the plan report."""
    from torch_helion.optimizer.legality import check_program

    _, m, args = _llama()
    res = _compile(m, args, tmp_path)
    notes = check_program(res.program).notes
    assert any("fp32 GEMM" in n for n in notes) and any("SIMT flash" in n for n in notes)
    plan_md = next(res.run_dir.rglob("plan.md")).read_text()
    assert "## Device paths" in plan_md and "SIMT flash" in plan_md
    _, m, args = _mamba(dtype=torch.bfloat16)
    notes = check_program(_compile(m, args, tmp_path / "m").program).notes
    assert any("three-pass scan" in n for n in notes)
    assert not any("GEMM" in n for n in notes)  # bf16 GEMMs of 256 rows take the CTA-pair kernel


def test_unknown_backend_raises():
    from torch_helion import CompileConfig, compile_model

    _, m, args = _llama()
    with pytest.raises(ValueError):
        compile_model(m, args, CompileConfig(backend="loom"))


def test_saved_artifact_round_trips(tmp_path):
    """compile_model(save_params=True) leaves 06_opir.json + params.pt; the
    Program read back is the same Program (the GPU test runs it)."""
    import torch

    from torch_helion import CompileConfig, compile_model
    from torch_helion.optimizer.opir import Program
    from workloads import configs
    from workloads.mamba import MambaConfig

    cfg = MambaConfig(batch=1, seq=256, d_model=64, headdim=32, d_state=32, chunk=128, n_layers=1, mode="chunked",
                      ngroups=1, use_conv=True, dtype=torch.float32)
    m = configs.build(cfg)
    (u,) = m.example_inputs(seed=1)
    res = compile_model(m, (u,), CompileConfig(run_name="a", results_dir=tmp_path, execute=False, save_params=True))
    prog = Program.from_json(tmp_path / "a" / "06_opir.json")
    assert prog.to_dict() == res.program.to_dict()
    params = torch.load(tmp_path / "a" / "params.pt", weights_only=True)
    assert set(prog.params) <= set(params)


def test_cost_model_calibration_recovers_known_terms():
    """The calibration fit recovers the efficiency and fixed cost that
    generated synthetic GEMM and elementwise timings."""
    from torch_helion.cost_models.b200 import B200Spec
    from torch_helion.cost_models.calibrate import fit

    hw = B200Spec()
    recs = []
    for waves, bn, k in ((1, 256, 768), (7, 256, 768), (3, 128, 1536), (194, 256, 4096), (40, 256, 14336)):
        work_us = waves * 128 * bn * k * 2 / (hw.sm_tflops * 1e12) * 1e6
        recs.append(dict(kind="gemm", dtype="bfloat16", waves=waves, tile_n=bn, K=k, measured_us=12.0 + work_us / 0.7))
    for nbytes in (1e7, 6e7, 3e8):
        recs.append(dict(kind="rmsnorm", dtype="bfloat16", bytes=nbytes,
                         measured_us=4.0 + nbytes / (hw.hbm_gbs * 1e9) * 1e6 / 0.5))
    got = fit(recs, hw)
    assert abs(got["eff_mma"] - 0.7) < 1e-6 and abs(got["gemm_fixed_us"] - 12.0) < 1e-6
    assert abs(got["eff_elem"] - 0.5) < 1e-6 and abs(got["elem_fixed_us"] - 4.0) < 1e-6
