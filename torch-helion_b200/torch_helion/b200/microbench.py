"""Time one C-ABI kernel on seeded synthetic operands.

    python -m torch_helion.b200.microbench attention --batch 1 --seq 4096 --hq 32 --hkv 8 --head-dim 128 --causal
    python -m torch_helion.b200.microbench ssd --batch 4 --seq 2048 --heads 24 --state 128
    python -m torch_helion.b200.microbench ssd-sweep --flush
    python -m torch_helion.b200.microbench gemm --m 8192 --n 3328 --k 768 --vs-torch
    python -m torch_helion.b200.microbench conv --batch 4 --seq 2048 --channels 1792
    python -m torch_helion.b200.microbench rmsnorm --m 8192 --k 768
    torchrun --nproc-per-node 8 -m torch_helion.b200.microbench allreduce --rows 32768 --cols 4096 --ctas 16,24,32

Each mode runs 3 warm-up launches and times ``--iters`` launches with CUDA
events (L2 flushed before each when ``--flush``), printing one JSON line with
the median time and the kernel's algorithmic throughput.  This is the
command behind the single-kernel ncu captures.

``allreduce`` (one process per GPU under torchrun) sums a bf16 [rows, cols] array
over the ranks with ``th_allreduce`` for every ``--ctas`` grid size and
with NCCL's ``all_reduce`` on the same bytes, checks that both give the
same sums, and prints rank 0's line: the max over ranks of each median
time and the algorithm bandwidth (bytes / time).

``ssd-sweep`` is the standalone chunked-scan sweep: batch 8, 64 heads of 64,
one B/C group, chunk 256, d_state in {64, 128, 256} x seqlen in {512, 2048,
8192, 16384}, no gate and no D skip; one JSON line per point.  Its bytes per
token are x in + y out (bf16), B and C (bf16) and dt (fp32, the ABI's dt
type), and the line carries the fraction of the measured HBM copy bandwidth
and of the measured bf16 tensor peak.
"""

from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import torch

from . import lib


def _time(fn, iters: int, flush: bool) -> float:
    buf = torch.empty(64 << 20, dtype=torch.float32, device="cuda") if flush else None
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        if buf is not None:
            buf.fill_(1.0)
        torch.cuda._sleep(200_000)  # keeps the GPU busy while the host enqueues the timed launch
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    ts.sort()
    return ts[len(ts) // 2] / 1e3  # seconds


def _ssd_case(batch: int, seq: int, h: int, n: int, gate: bool, p: int = 64):
    """th_ssd on seeded operands: x, B, C ~ N(0, 1) bf16, dt log-uniform in
    [1e-3, 0.1], A = -exp(U[0, log 16]).  Returns (launch, algorithmic bytes)."""
    dev, bf = "cuda", torch.bfloat16
    t = batch * seq
    x = torch.randn(t, h * p, device=dev).to(bf)
    B = torch.randn(t, n, device=dev).to(bf)
    C = torch.randn(t, n, device=dev).to(bf)
    dt = torch.exp(torch.rand(t, h, device=dev) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3))
    A = -torch.exp(torch.rand(h, device=dev) * math.log(16.0))
    D = torch.ones(h, device=dev) if gate else None
    z = torch.randn(t, h * p, device=dev).to(bf) if gate else None
    out = torch.empty(t, h * p, device=dev, dtype=bf)
    gss = torch.empty(t, h, device=dev) if gate else None
    ws = torch.empty(lib.ssd_workspace_size(batch, seq, h, p, n, 256), dtype=torch.uint8, device=dev)
    fn = lambda: lib.ssd(x, dt, A, B, C, out, batch=batch, seq=seq, heads=h, head_dim=p, ngroups=1,
                         state_dim=n, chunk=256, D=D, z=z, gss=gss, workspace=ws)
    per_tok = 2 * h * p * 2 + 2 * n * 2 + 4 * h          # x in, y out, B, C, dt
    per_tok += (h * p * 2 + 4 * h) if gate else 0         # z in, per-head sum of squares out
    return fn, t * per_tok


def _ssd_sweep(a) -> None:
    peaks_file = Path(__file__).resolve().parents[3] / "MEASURED_PEAKS.json"
    peaks = json.loads(peaks_file.read_text()) if peaks_file.exists() else {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
    src = "measured" if peaks_file.exists() else "fallback"
    h, p, batch, L = 64, 64, 8, 256
    for n in (64, 128, 256):
        for seq in (512, 2048, 8192, 16384):
            fn, nbytes = _ssd_case(batch, seq, h, n, gate=False)
            sec = _time(fn, a.iters, a.flush)
            t = batch * seq
            flops = t * h * (2 * L * p + 4 * p * n + 2 * L * n / h)
            gbs, tfs = nbytes / sec / 1e9, flops / sec / 1e12
            ridge = peaks["bf16_tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9)
            print(json.dumps({"kernel": "ssd", "batch": batch, "heads": h, "head_dim": p, "state": n, "seq": seq,
                              "us": sec * 1e6, "bytes": nbytes, "flops": flops, "GB/s": gbs,
                              "hbm_frac": gbs / peaks["hbm_gbs"], "TFLOP/s": tfs,
                              "tensor_frac": tfs / peaks["bf16_tflops"],
                              "bound": "hbm" if flops / nbytes < ridge else "tensor", "peaks": src,
                              "device_error": lib.device_error()}), flush=True)
            del fn
            torch.cuda.empty_cache()


def _allreduce(a) -> None:
    import os
    from datetime import timedelta

    import torch.distributed as dist

    from .collectives import SymmetricRows, multimem_available

    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        if not multimem_available(dev):
            raise lib.B200KernelError("no multicast symmetric memory on this node")
        sym = SymmetricRows(a.rows, a.cols, torch.bfloat16, dev)
        g = torch.Generator(device=dev).manual_seed(dist.get_rank())
        src = torch.randn(a.rows, a.cols, device=dev, generator=g).to(torch.bfloat16)
        ref = src.clone()
        dist.all_reduce(ref)
        sym.buf.copy_(src)
        torch.cuda.synchronize()
        dist.barrier()
        sym.allreduce_rows(0, a.rows)
        torch.cuda.synchronize()
        same = bool(torch.equal(sym.buf, ref))
        nbytes = a.rows * a.cols * 2

        def med(fn) -> float:  # median device time, max over ranks
            t = torch.tensor([_time(fn, a.iters, False)], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t)

        rows = {"nccl": med(lambda: dist.all_reduce(ref))}
        for c in (int(v) for v in a.ctas.split(",")):
            sym.ctas = c
            rows[f"th_allreduce ctas={c}"] = med(lambda: sym.allreduce_rows(0, a.rows))
        err = lib.device_error()
        if dist.get_rank() == 0:
            print(json.dumps({"kernel": "allreduce", "ranks": dist.get_world_size(), "bytes": nbytes,
                              "same_sums_as_nccl": same, "device_error": err,
                              "us": {k: v * 1e6 for k, v in rows.items()},
                              "algbw_gbs": {k: nbytes / v / 1e9 for k, v in rows.items()}}))
        torch.cuda.synchronize()
        dist.barrier()
        del sym
    finally:
        dist.destroy_process_group()


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("kernel", choices=["attention", "ssd", "ssd-sweep", "gemm", "conv", "rmsnorm", "rowstat",
                                       "allreduce"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--hq", type=int, default=32)
    ap.add_argument("--hkv", type=int, default=8)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--causal", action="store_true")
    ap.add_argument("--heads", type=int, default=24)
    ap.add_argument("--state", type=int, default=128)
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=3328)
    ap.add_argument("--k", type=int, default=768)
    ap.add_argument("--channels", type=int, default=1792)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--ctas", default="16,24,32", help="allreduce: th_allreduce grid sizes to time")
    # (not --m / --k: under torchrun those would be taken for abbreviations of its own options)
    ap.add_argument("--rows", type=int, default=32768, help="allreduce: rows of the bf16 array")
    ap.add_argument("--cols", type=int, default=4096, help="allreduce: columns of the bf16 array")
    ap.add_argument("--flush", action="store_true")
    ap.add_argument("--no-gate", action="store_true", help="ssd: no silu(z) gate, no D skip, no row sums")
    ap.add_argument("--vs-torch", action="store_true", help="gemm: also time torch.matmul (cuBLAS)")
    ap.add_argument("--residual", action="store_true", help="gemm: add a residual [m, n] in the epilogue")
    ap.add_argument("--swiglu", action="store_true",
                    help="gemm: row-scaled SwiGLU epilogue (gate/up interleaved in 64-column blocks), output [m, n/2]")
    a = ap.parse_args(argv)
    torch.manual_seed(0)
    dev, bf = "cuda", torch.bfloat16
    extra: dict = {}
    if a.kernel == "ssd-sweep":
        _ssd_sweep(a)
        return
    if a.kernel == "allreduce":
        _allreduce(a)
        return
    if a.kernel == "attention":
        t = a.batch * a.seq
        q = torch.randn(t, a.hq * a.head_dim, device=dev).to(bf)
        k = torch.randn(t, a.hkv * a.head_dim, device=dev).to(bf)
        v = torch.randn(t, a.hkv * a.head_dim, device=dev).to(bf)
        o = torch.empty_like(q)
        fn = lambda: lib.attention(q, k, v, o, batch=a.batch, seq=a.seq, hq=a.hq, hkv=a.hkv, head_dim=a.head_dim,
                                   scale=a.head_dim ** -0.5, causal=a.causal)
        work, unit = 4.0 * a.batch * a.hq * a.seq * a.seq * a.head_dim * (0.5 if a.causal else 1.0), "TFLOP/s"
    elif a.kernel == "ssd":
        fn, work = _ssd_case(a.batch, a.seq, a.heads, a.state, gate=not a.no_gate)
        unit = "GB/s"
    elif a.kernel == "gemm":
        x = torch.randn(a.m, a.k, device=dev).to(bf)
        w = (torch.randn(a.n, a.k, device=dev) * 0.02).to(bf)
        d = torch.empty(a.m, a.n // 2 if a.swiglu else a.n, device=dev, dtype=bf)
        if a.residual:  # the row-parallel projections' epilogue: + residual
            res = torch.randn(a.m, a.n, device=dev).to(bf)
            fn = lambda: lib.gemm(x, w, d, residual=res)
        elif a.swiglu:  # the MLP's gate|up epilogue: RMSNorm row scale from 64-column partial sums, SwiGLU
            parts = torch.rand(a.m, (a.k + 63) // 64, device=dev) * 64.0
            fn = lambda: lib.gemm(x, w, d, rs_parts=parts, rs_inv_k=1.0 / a.k, rs_eps=1e-5, swiglu=True)
        else:
            fn = lambda: lib.gemm(x, w, d)
        work, unit = 2.0 * a.m * a.n * a.k, "TFLOP/s"
        if a.vs_torch:  # cuBLAS through torch on the same operands, for comparison
            extra["torch_us"] = _time(lambda: torch.matmul(x, w.t()), a.iters, a.flush) * 1e6
    elif a.kernel in ("rmsnorm", "rowstat"):  # --m rows x --k columns
        x = torch.randn(a.m, a.k, device=dev).to(bf)
        if a.kernel == "rmsnorm":
            g = torch.rand(a.k, device=dev) + 0.5
            y = torch.empty_like(x)
            fn = lambda: lib.rmsnorm(x, g, 1e-5, out=y)
            work = 2.0 * a.m * a.k * 2
        else:
            s_out = torch.empty(a.m, device=dev)
            fn = lambda: lib.rowstat(x, out=s_out)
            work = a.m * a.k * 2 + a.m * 4.0
        unit = "GB/s"
    else:
        t = a.batch * a.seq
        x = torch.randn(t, a.channels, device=dev).to(bf)
        w = torch.randn(a.channels, 4, device=dev)
        y = torch.empty_like(x)
        fn = lambda: lib.conv1d(x, w, y, batch=a.batch, seq=a.seq, act=lib.ACT_SILU)
        work, unit = 2.0 * t * a.channels * 2, "GB/s"
    sec = _time(fn, a.iters, a.flush)
    rate = work / sec / (1e12 if unit == "TFLOP/s" else 1e9)
    print(json.dumps({"kernel": a.kernel, "args": vars(a), "us": sec * 1e6, "rate": rate, "unit": unit, **extra,
                      "device_error": lib.device_error()}))


if __name__ == "__main__":
    main()
