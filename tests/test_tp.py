"""Tensor parallelism of the Llama block (heads / FFN columns, one NCCL
all-reduce after o_proj and after down_proj).

CPU tests run the sharded programs in the fp64 OpIR interpreter
(``oracle.interpret``): once in lockstep in one process, once as two gloo
ranks that sum their partials with ``dist.all_reduce``, and compare with the
unsharded program and the eager oracle.  The GPU test runs two NCCL ranks
through ``compile_model(world_size=2)`` and needs two devices.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import REPO, rel_l2
from oracle import interpret as I
from oracle import models as O

SMALL = dict(batch=2, seq=32, hidden=128, heads=4, kv_heads=2, intermediate=256, causal=True, dtype=torch.float32)


def _program(tmp_path, **kw):
    from torch_helion import CompileConfig, compile_model
    from workloads.llama_block import LlamaBlockConfig, build_llama_block

    cfg = LlamaBlockConfig(**{**SMALL, **kw})
    m = build_llama_block(cfg, 0)
    (x,) = m.example_inputs(seed=1)
    res = compile_model(m, (x,), CompileConfig(run_name="tp", results_dir=tmp_path, execute=False))
    ref = O.llama_block_forward({k: v.detach() for k, v in m.state_dict().items()}, x, heads=cfg.heads,
                                kv_heads=cfg.kv_heads, eps=cfg.eps, rope_theta=cfg.rope_theta, causal=cfg.causal,
                                model_dtype=cfg.dtype)
    return res.program, res.graph.params, x, ref


def _lockstep(shards, x):
    """Run every rank's program kernel by kernel, summing tp_allreduce outputs."""
    envs = []
    for prog, params in shards:
        env = {prog.inputs[0]: x.reshape(prog.tensors[prog.inputs[0]].shape).double()}
        env.update({n: params[n].double() for n in prog.params})
        envs.append(env)
    n_k = len(shards[0][0].kernels)
    assert all(len(p.kernels) == n_k for p, _ in shards)
    for i in range(n_k):
        outs = [I.run_kernel(p.kernels[i], env) for (p, _), env in zip(shards, envs)]
        if shards[0][0].kernels[i].attrs.get("tp_allreduce"):
            total = {t: sum(o[t] for o in outs) for t in outs[0]}
            outs = [dict(total) for _ in outs]
        for env, o in zip(envs, outs):
            env.update(o)
    prog = shards[0][0]
    return envs[0][prog.outputs[0]].reshape(x.shape)


@pytest.mark.parametrize("rows,n", [(32768, 4), (32768, 8), (8192, 3), (1000, 4), (256, 2), (384, 3)])
def test_chunk_bounds_cover_rows_in_whole_tiles(rows, n):
    """The tensor-parallel tail's row chunks: contiguous, covering every row
    once, every boundary on a 128-row GEMM tile, no empty chunk, and with
    three or more chunks the first and last about half as tall as the rest."""
    from torch_helion.b200.runtime import _chunk_bounds

    b = _chunk_bounds(rows, n)
    assert len(b) == n and b[0][0] == 0 and b[-1][1] == rows
    assert all(r1 == s0 for (_, r1), (s0, _) in zip(b, b[1:]))
    assert all(r0 < r1 and r0 % 128 == 0 for r0, r1 in b)
    if n >= 3 and rows >= 128 * 4 * n:
        mid = [r1 - r0 for r0, r1 in b[1:-1]]
        for r0, r1 in (b[0], b[-1]):
            assert abs((r1 - r0) - min(mid) / 2) <= 128


def test_shard_structure(tmp_path):
    from torch_helion.b200.tp import shard_program

    prog, params, _, _ = _program(tmp_path)
    s0, p0 = shard_program(prog, params, 2, 0)
    s1, p1 = shard_program(prog, params, 2, 1)
    att = [k for k in s0.kernels if k.kind == "attention"][0]
    assert (att.attrs["heads"], att.attrs["kv_heads"]) == (2, 1)
    marked = [k.name for k in s0.kernels if k.attrs.get("tp_allreduce")]
    assert len(marked) == 2  # o_proj and down_proj
    # rank 1 adds no residual: its row-parallel kernels read only their LHS
    for k in s1.kernels:
        if k.attrs.get("tp_allreduce"):
            assert not [a for a in k.args if a.role == "extra"], k
    # the sharded weights are column/row blocks of the originals
    for name in s1.params:
        if "@tp1/2" in name:
            base = name.split("@tp")[0]
            w, ws = params[base], p1[name]
            assert ws.numel() * 2 == w.numel()
    # the unsharded program is untouched
    assert [k.attrs.get("heads") for k in prog.kernels if k.kind == "attention"] == [4]


@pytest.mark.parametrize("world,kw", [(2, {}), (4, dict(heads=8, kv_heads=4)), (2, dict(kv_heads=4))],
                         ids=["gqa_w2", "gqa_w4", "mha_w2"])
def test_lockstep_matches_unsharded(tmp_path, world, kw):
    from torch_helion.b200.tp import shard_program

    prog, params, x, ref = _program(tmp_path, **kw)
    full = I.program_outputs(prog, params, [x])[0].reshape(x.shape)
    assert rel_l2(full, ref) < 1e-6  # the eager oracle runs in the model dtype (fp32)
    shards = [shard_program(prog, params, world, r) for r in range(world)]
    out = _lockstep(shards, x)
    assert rel_l2(out, full) < 1e-12


def test_rejects_indivisible(tmp_path):
    from torch_helion.b200.tp import TPError, shard_program

    prog, params, _, _ = _program(tmp_path)
    with pytest.raises(TPError):
        shard_program(prog, params, 3, 0)


def test_rejects_mamba(tmp_path):
    from torch_helion import CompileConfig, compile_model
    from torch_helion.b200.tp import TPError, shard_program
    from workloads.mamba import MambaConfig, build_mamba_model

    m = build_mamba_model(MambaConfig(batch=1, seq=64, d_model=64, expand=2, headdim=16, d_state=16, chunk=32,
                                      n_layers=1, mode="chunked", dtype=torch.float32), 0)
    args = m.example_inputs(1)
    res = compile_model(m, args, CompileConfig(run_name="m", results_dir=tmp_path, execute=False))
    with pytest.raises(TPError):
        shard_program(res.program, res.graph.params, 2, 0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, path, prog_dict, params, x):
    import sys

    for p in (str(REPO / "torch-helion_b200"), str(REPO)):
        if p not in sys.path:
            sys.path.insert(0, p)
    from oracle import interpret as I2
    from torch_helion.b200.tp import shard_program
    from torch_helion.optimizer.opir import Program

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        prog = Program.from_dict(prog_dict)
        sp, spar = shard_program(prog, params, world, rank)
        out = I2.program_outputs(sp, spar, [x], allreduce=lambda t: dist.all_reduce(t))[0]
        torch.save(out, f"{path}/rank{rank}.pt")
    finally:
        dist.destroy_process_group()


def test_gloo_world2(tmp_path):
    prog, params, x, ref = _program(tmp_path)
    full = I.program_outputs(prog, params, [x])[0].reshape(x.shape)
    used = {n: params[n] for n in prog.params}
    mp.start_processes(_gloo_rank, args=(2, _free_port(), str(tmp_path), prog.to_dict(), used, x), nprocs=2,
                       start_method="spawn")
    outs = [torch.load(tmp_path / f"rank{r}.pt").reshape(x.shape) for r in range(2)]
    assert torch.equal(outs[0], outs[1])  # every rank holds the full result
    assert rel_l2(outs[0], full) < 1e-12
    assert rel_l2(outs[0], ref) < 1e-6


# ------------------------------------------------------- GPU, one device
@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_row_chunked_schedule_matches_sequential(tmp_path, dtype):
    """The row-chunked tensor-parallel schedule (all-reduce of chunk c on a
    second stream overlapping chunk c+1's GEMMs) computes exactly what the
    launch-by-launch order computes.  Rank 0 of a 2-way shard runs on one GPU
    with a stand-in all-reduce (x2: two ranks holding the same partial)."""
    from torch_helion.b200.runtime import CompiledProgram
    from torch_helion.b200.tp import shard_program

    prog, params, x, _ = _program(tmp_path, batch=2, seq=256, hidden=512, heads=8, kv_heads=4, intermediate=1024,
                                  dtype=dtype)
    sp, spar = shard_program(prog, params, 2, 0)
    outs = []
    for chunks in (1, 4):
        mod = CompiledProgram(sp, spar, "cuda:0", tp_rank=0, tp_world=2, allreduce=lambda t: t.mul_(2.0),
                              tp_chunks=chunks)
        assert (mod._pipe is not None) == (chunks > 1)
        outs.append(mod(x.to("cuda:0"))[0].float().cpu())
        torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


# ------------------------------------------------------------------ GPU (NCCL)
def _nccl_rank(rank, world, port, path, kw):
    import sys

    for p in (str(REPO / "torch-helion_b200"), str(REPO)):
        if p not in sys.path:
            sys.path.insert(0, p)
    from datetime import timedelta

    from torch_helion import CompileConfig, compile_model
    from workloads.llama_block import LlamaBlockConfig, build_llama_block

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        cfg = LlamaBlockConfig(**kw)
        m = build_llama_block(cfg, 0)
        (x,) = m.example_inputs(seed=1)
        res = compile_model(m, (x,), CompileConfig(run_name=f"tp{rank}", results_dir=path, device=f"cuda:{rank}",
                                                   world_size=world, tp_mode="heads", reference_check=False,
                                                   verify_passes=False, tp_allreduce="nccl"))
        out = res.run(x.to(f"cuda:{rank}"))[0].float().cpu()
        torch.cuda.synchronize()
        torch.save(out, f"{path}/rank{rank}.pt")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("kw", [
    dict(batch=2, seq=128, hidden=512, heads=8, kv_heads=2, intermediate=1024, causal=True, dtype=torch.float32),
    dict(batch=2, seq=256, hidden=1024, heads=8, kv_heads=4, intermediate=2048, causal=True, dtype=torch.bfloat16),
], ids=["fp32", "bf16"])
def test_nccl_world2(tmp_path, kw):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from workloads.llama_block import LlamaBlockConfig, build_llama_block

    mp.start_processes(_nccl_rank, args=(2, _free_port(), str(tmp_path), kw), nprocs=2, start_method="spawn")
    cfg = LlamaBlockConfig(**kw)
    m = build_llama_block(cfg, 0)
    (x,) = m.example_inputs(seed=1)
    ref = O.llama_block_forward({k: v.detach() for k, v in m.state_dict().items()}, x, heads=cfg.heads,
                                kv_heads=cfg.kv_heads, eps=cfg.eps, rope_theta=cfg.rope_theta, causal=cfg.causal,
                                model_dtype=cfg.dtype)
    outs = [torch.load(tmp_path / f"rank{r}.pt").reshape(x.shape) for r in range(2)]
    tol = 1e-5 if cfg.dtype == torch.float32 else 2e-2
    for o in outs:
        assert rel_l2(o, ref) < tol


def test_rejects_qkv_from_one_accumulator(tmp_path):
    """A program whose q and k are both outputs of ONE accumulator (one wide
    GEMM split by columns, as a reference-built OpIR may have it) cannot be
    sharded by contiguous column blocks: shard_program refuses it."""
    import copy

    from torch_helion.b200.tp import TPError, shard_program

    prog, params, _, _ = _program(tmp_path)
    prog = copy.deepcopy(prog)
    att = next(k for k in prog.kernels if k.kind == "attention")
    q_t, k_t = next(a.tensor for a in att.args if a.role == "q"), next(a.tensor for a in att.args if a.role == "k")
    qkv = next(k for k in prog.kernels if any(o.tensor == q_t for o in k.outputs))
    q_out = next(o for o in qkv.outputs if o.tensor == q_t)
    k_out = next(o for o in qkv.outputs if o.tensor == k_t)
    k_out.value = q_out.value  # k now reads q's accumulator
    with pytest.raises(TPError, match="one accumulator"):
        shard_program(prog, params, 2, 0)
