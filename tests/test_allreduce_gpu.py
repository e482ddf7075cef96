"""th_allreduce: the in-place multicast all-reduce of the tensor-parallel block.

* two ranks (two GPUs): random bf16 / fp32 rows reduced chunk by chunk, as
  the row-chunked schedule calls it, against the fp32 sum of the gathered
  inputs; and the tensor-parallel Llama block with ``tp_allreduce="multimem"``
  against the eager oracle (``test_tp.py`` runs the same block over NCCL);
* a rank that never calls: the other rank's handshake gives up after the
  bounded wait, reports TH_DEVERR_MBAR_TIMEOUT through the device error word
  and leaves its data untouched.
"""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import REPO, rel_l2
from oracle import models as O

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(rank: int, world: int, port: int) -> None:
    import sys

    for p in (str(REPO / "torch-helion_b200"), str(REPO)):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))


def _multicast_ok() -> bool:
    from torch.distributed import _symmetric_memory as symm

    try:
        return bool(symm._SymmetricMemory.has_multicast_support(symm.DeviceType.CUDA, 0))
    except Exception:
        return False


def _rows_rank(rank, world, port, path, dtype_name, stats=False):
    _setup(rank, world, port)
    try:
        from torch_helion.b200 import lib
        from torch_helion.b200.collectives import SymmetricRows

        dtype = getattr(torch, dtype_name)
        dev = torch.device("cuda", rank)
        rows, cols = 1024, 4096
        sym = SymmetricRows(rows, cols, dtype, dev, ctas=24)
        sym.stats = stats
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        src = torch.randn(rows, cols, device=dev, generator=g).to(dtype)
        sym.buf.copy_(src)
        everyone = [torch.empty_like(src) for _ in range(world)]
        dist.all_gather(everyone, src)
        torch.cuda.synchronize()
        for r0, r1 in ((0, 256), (256, 512), (512, 1024)):  # chunk by chunk, in place
            sym.allreduce_rows(r0, r1)
        torch.cuda.synchronize()
        err = lib.device_error()
        want = torch.stack([e.float() for e in everyone]).sum(0).to(dtype)
        torch.save({"err": err, "got": sym.buf.float().cpu(), "want": want.float().cpu(),
                    "sumsq": sym.sumsq.cpu() if stats else None}, f"{path}/rank{rank}.pt")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("dtype_name,stats", [("bfloat16", False), ("float32", False), ("bfloat16", True)],
                         ids=["bf16", "fp32", "bf16-rowstats"])
def test_allreduce_world2(tmp_path, dtype_name, stats):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    if not _multicast_ok():
        pytest.skip("no multicast symmetric memory on this node")
    mp.start_processes(_rows_rank, args=(2, _free_port(), str(tmp_path), dtype_name, stats), nprocs=2,
                       start_method="spawn")
    res = [torch.load(tmp_path / f"rank{r}.pt") for r in range(2)]
    for r in res:
        assert r["err"] == 0
        # the switch adds the ranks' values in fp32 and rounds the sum once to the buffer's type; its
        # rounding of that last step need not be round-to-nearest-even, so allow one unit in the last
        # place of the type (bf16: 8 significant bits, fp32: 24)
        ulp = 2.0 ** -7 if dtype_name == "bfloat16" else 2.0 ** -23
        assert torch.allclose(r["got"], r["want"], rtol=ulp, atol=1e-30)
    assert torch.equal(res[0]["got"], res[1]["got"])  # every rank holds the same sums
    if stats:  # each row's sum of squares of the reduced values, on every rank
        want_ss = (res[0]["got"].double() ** 2).sum(1)
        for r in res:
            assert torch.allclose(r["sumsq"].double(), want_ss, rtol=1e-5, atol=0)


def _block_rank(rank, world, port, path, kw):
    _setup(rank, world, port)
    try:
        from torch_helion import CompileConfig, compile_model
        from workloads.llama_block import LlamaBlockConfig, build_llama_block

        cfg = LlamaBlockConfig(**kw)
        m = build_llama_block(cfg, 0)
        (x,) = m.example_inputs(seed=1)
        res = compile_model(m, (x,), CompileConfig(run_name=f"mm{rank}", results_dir=path, device=f"cuda:{rank}",
                                                   world_size=world, tp_mode="heads", reference_check=False,
                                                   verify_passes=False, tp_allreduce="multimem", tp_chunks=2))
        assert res.module._multimem
        # the second RMSNorm's statistic comes from the all-reduce: one row-statistics launch is left
        assert sum(n.startswith("rowstat(") for n in res.module.launch_names()) == 1
        out = res.run(x.to(f"cuda:{rank}"))[0].float().cpu()
        torch.cuda.synchronize()
        torch.save(out, f"{path}/rank{rank}.pt")
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_llama_block_multimem_world2(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    if not _multicast_ok():
        pytest.skip("no multicast symmetric memory on this node")
    from workloads.llama_block import LlamaBlockConfig, build_llama_block

    kw = dict(batch=2, seq=256, hidden=1024, heads=8, kv_heads=4, intermediate=2048, causal=True, dtype=torch.bfloat16)
    mp.start_processes(_block_rank, args=(2, _free_port(), str(tmp_path), kw), nprocs=2, start_method="spawn")
    cfg = LlamaBlockConfig(**kw)
    m = build_llama_block(cfg, 0)
    (x,) = m.example_inputs(seed=1)
    ref = O.llama_block_forward({k: v.detach() for k, v in m.state_dict().items()}, x, heads=cfg.heads,
                                kv_heads=cfg.kv_heads, eps=cfg.eps, rope_theta=cfg.rope_theta, causal=cfg.causal,
                                model_dtype=cfg.dtype)
    outs = [torch.load(tmp_path / f"rank{r}.pt").reshape(x.shape) for r in range(2)]
    assert torch.equal(outs[0], outs[1])
    assert rel_l2(outs[0], ref) < 2e-2


def _timeout_rank(rank, world, port, path):
    _setup(rank, world, port)
    try:
        from torch_helion.b200 import lib
        from torch_helion.b200.collectives import SymmetricRows

        dev = torch.device("cuda", rank)
        sym = SymmetricRows(64, 256, torch.bfloat16, dev, ctas=1)
        sym.buf.fill_(1.5 + rank)
        torch.cuda.synchronize()
        lib.device_error(clear=True)
        if rank == 0:  # rank 1 never calls: rank 0's handshake waits for a signal that nothing sends
            sym.allreduce_rows(0, 64)
            torch.cuda.synchronize()
            err = lib.device_error(clear=True)
            torch.save({"err": err, "untouched": bool((sym.buf == 1.5).all().item())}, f"{path}/timeout.pt")
        dist.barrier()  # rank 1 keeps its buffer mapped until rank 0 is done
    finally:
        dist.destroy_process_group()


def test_allreduce_handshake_times_out(tmp_path):
    """A rank that never joins: the other rank's all-reduce gives up after the bounded wait (2 s),
    sets TH_DEVERR_MBAR_TIMEOUT and leaves its data as it was."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    if not _multicast_ok():
        pytest.skip("no multicast symmetric memory on this node")
    mp.start_processes(_timeout_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    r = torch.load(tmp_path / "timeout.pt")
    assert r["err"] & 1  # TH_DEVERR_MBAR_TIMEOUT
    assert r["untouched"]
