"""Benchmark: tokens/sec per forward of the compiled model on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c3|c2|c4|c1]

Default workload: BASELINE config C3, the Llama-3-8B-geometry decoder block
in bf16 (B8 S4096 D4096 Hq32 Hkv8 F14336, causal) through compile_model ->
th_* kernels.  At N=1 the whole block runs on one GPU; with N > 1 (torchrun,
one rank per GPU) the same B8 S4096 block runs tensor-parallel over the N
ranks (heads and FFN columns, one NCCL all-reduce after o_proj and one after
down_proj), so the scaling is strong and ``value`` is the job's tokens/s.
``--workload c4`` splits the 24-layer Mamba-2 backbone's batch of 16 over
the ranks (no communication, strong scaling); ``--workload c2`` runs one
Mamba-2 block batch per GPU (weak scaling).

One JSON line on rank 0:
  value       tokens/s, inputs resident in HBM, L2 flushed between steps,
              device time from CUDA events (max over ranks)
  e2e         the same forward through the public serving entry
              (CompileResult.streaming_runner) with pinned HOST buffers: the
              H2D of every step's input and the D2H of its output are inside
              the timed region, overlapped with neighbouring forwards; under
              tensor parallelism each rank moves only its own rows
  roofline    the dominant kernel's algorithmic bytes (or flops) per launch
              (of this rank's shard) / its event-timed duration, against
              MEASURED_PEAKS.json
  cpu_baseline the CPU oracle (the reference's eager forward restated in
              oracle/) timed on this host (rank 0, N=1 only)
``--impl reference`` prints the reference arm: that CPU forward alone, on the
same workload, on all host threads.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "torch-helion_b200"))
sys.path.insert(0, str(REPO))

L2_FLUSH_BYTES = 256 << 20


def _peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def _workload(name: str, rank: int, world: int = 1):
    """(cfg, model, this rank's input, description, scaling).  C3 runs the
    whole B8 S4096 block, tensor-parallel over the ranks at N > 1 (strong
    scaling); C4 splits the batch of 16 across the ranks (strong scaling);
    C2 runs one full C2 batch per GPU (weak scaling)."""
    from workloads import configs

    scaling, seed = "weak", 1 + rank
    if name == "c2":
        cfg = configs.c2_mamba_block_bf16()
        desc = "C2 Mamba-2 block bf16: B4 S2048 d768 expand2 headdim64 (24 heads) d_state128 ngroups1 conv4 chunk256"
    elif name == "c4":
        if 16 % world:
            raise SystemExit("c4 splits batch 16: use 1, 2, 4 or 8 GPUs")
        cfg = configs.c4_mamba24_bf16(batch=16 // world)
        desc = (f"C4 Mamba-2 24-layer backbone bf16 B16 S2048 d1024 d_state128 chunk256, vocab 50280 embedding, "
                f"final RMSNorm" + (f"; batch split {16 // world} per GPU" if world > 1 else ""))
        scaling = "strong"
    elif name == "c1":
        cfg = configs.c1_llama_fp32()
        desc = "C1 Llama block fp32: B1 S128 D512 H8 KV8 d64 F1408 causal"
    elif name == "c3":
        cfg = configs.c3_llama8b_bf16(batch=8, seq=4096)
        desc = ("C3 Llama-3-8B-geometry block bf16 B8 S4096 D4096 Hq32 Hkv8 d128 F14336 theta5e5 causal"
                + (f", tensor-parallel over {world} GPUs" if world > 1 else ""))
        scaling, seed = "strong", 1  # every rank holds the same batch
    else:
        raise SystemExit(f"unknown workload {name}")
    model = configs.build(cfg, seed=0)
    (x,) = model.example_inputs(seed=seed)
    return cfg, model, x, desc, scaling


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 100 ms while the GPU works."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int) -> None:
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = [r for r in self.rows if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        num = lambda v: float(v) if v.replace(".", "", 1).isdigit() else None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        pw = [num(r[3]) for r in rows if num(r[3]) is not None]
        # samples under load: the GPU drawing well above idle power
        busy = [float(r[1]) for r in rows if num(r[1]) is not None and num(r[3]) is not None and num(r[3]) > 250.0]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(busy or sm) if (busy or sm) else None,
                "sm_max_mhz": num(rows[0][2]), "reasons": reasons, "samples": len(rows),
                "samples_under_load": len(busy), "power_w_max": max(pw) if pw else None}


def kernel_work(launch, prog, module) -> dict:
    """Algorithmic bytes and flops of one launch of THIS rank's program (what
    the kernel must move / compute, not what it happens to move).  GEMM
    widths come from the (possibly tensor-parallel-sharded) weights."""
    name, kind = launch.name, launch.kind
    spec = next((k for k in prog.kernels if k.name == name), None)
    eb = 2 if module.dtype != torch.float32 else 4
    if kind == "rowstat":
        t = module.views[name[len("rowstat("):-1]]
        return {"bytes": t.numel() * eb + t.shape[0] * 4, "flops": 2.0 * t.numel()}
    if spec is None:
        return {"bytes": 0, "flops": 0}
    a = spec.attrs
    if kind == "gemm":
        T = spec.grid["rows"]
        rhs = [prog.tensors[x.tensor].shape for x in spec.args if x.role == "rhs"]
        K = rhs[0][0]
        N = sum(r[1] for r in rhs)  # sibling GEMMs (q|k|v, gate|up) share the LHS: their widths add
        out = sum(prog.tensors[o.tensor].numel for o in spec.outputs) * eb
        extra = sum(prog.tensors[x.tensor].numel * eb for x in spec.args if x.role == "extra")
        return {"bytes": T * K * eb + N * K * eb + out + extra, "flops": 2.0 * T * N * K}
    if kind == "ssd":
        T = a["batch"] * a["seq"]
        H, P, G, N = a["heads"], a["head_dim"], a["ngroups"], a["state_dim"]
        per_tok = 2 * H * P * eb + 2 * G * N * eb + 4 * H          # x in, y out, B, C, dt (fp32)
        per_tok += H * P * eb if a.get("gate") else 0               # z gate read
        per_tok += 4 * H                                            # gss out
        L = min(256, a["seq"])
        flops = T * H * (2 * L * P + 4 * P * N + 2 * L * N / max(1, H // G))
        return {"bytes": T * per_tok, "flops": flops}
    if kind == "causal_conv1d":
        t = prog.tensors[spec.outputs[0].tensor]
        return {"bytes": 2 * t.numel * eb, "flops": 2.0 * a["width"] * t.numel}
    if kind == "attention":
        b, s, h, d = a["batch"], a["seq"], a["heads"], a["head_dim"]
        return {"bytes": (2 * b * s * h * d + 2 * b * s * a.get("kv_heads", h) * d) * eb,
                "flops": 4.0 * b * h * s * s * d * (0.5 if a.get("causal") else 1.0)}
    t = prog.tensors[spec.outputs[0].tensor]
    return {"bytes": 2 * t.numel * eb, "flops": 3.0 * t.numel}


def _eager_forward(cfg, model):
    """The reference's eager forward as restated in the oracle, in the model
    dtype, as a function of the input batch."""
    from oracle import models as O

    sd = {k: v.detach() for k, v in model.state_dict().items()}
    dt = cfg.dtype
    if hasattr(cfg, "d_state"):
        return lambda xb: O.mamba_forward(sd, xb, n_layers=cfg.n_layers, d_model=cfg.d_model, expand=cfg.expand,
                                          headdim=cfg.headdim, d_state=cfg.d_state, ngroups=cfg.ngroups,
                                          chunk=cfg.chunk, eps=cfg.eps, use_conv=cfg.use_conv, d_conv=cfg.d_conv,
                                          mode=cfg.mode, embedding=cfg.vocab is not None, lm_head=cfg.tie_lm_head,
                                          dtype=dt)
    return lambda xb: O.llama_block_forward(sd, xb, heads=cfg.heads, kv_heads=cfg.kv_heads, eps=cfg.eps,
                                            rope_theta=cfg.rope_theta, causal=cfg.causal, model_dtype=dt, dtype=dt)


def _sample_rows(fwd, x, budget_s: float) -> tuple[torch.Tensor, float]:
    """The largest leading batch slice of ``x`` whose forward fits ``budget_s``
    (the whole batch when it does), and one forward's time on it."""
    b = x.shape[0]
    t0 = time.perf_counter()
    fwd(x[:1])
    t1 = time.perf_counter() - t0
    rows = max(1, min(b, int(budget_s / max(t1, 1e-4))))
    if rows == 1:
        return x[:1], t1
    t0 = time.perf_counter()
    fwd(x[:rows])
    return x[:rows], time.perf_counter() - t0


def cpu_baseline(cfg, model, x, budget_s: float = 20.0) -> dict:
    """The reference's eager forward, as restated in the oracle, on this host:
    the whole workload batch when a forward takes at most a quarter of the
    budget, else the largest batch slice that does; median of the repeats
    that fit the budget."""
    torch.set_num_threads(os.cpu_count() or 1)
    fwd = _eager_forward(cfg, model)
    with torch.no_grad():
        xb, once = _sample_rows(fwd, x, budget_s / 4)
        reps = max(1, min(20, int(budget_s / max(once, 1e-3))))
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fwd(xb)
            ts.append(time.perf_counter() - t0)
    med = statistics.median(ts)
    tokens = xb.shape[0] * xb.shape[1]
    whole = "the whole workload batch" if xb.shape[0] == x.shape[0] else f"batch {xb.shape[0]} of {x.shape[0]}"
    return {"value": tokens / med, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": (f"oracle eager forward in {str(cfg.dtype).replace('torch.', '')} ({whole}: "
                       f"{xb.shape[0]} x seq {xb.shape[1]}); median of {reps} after 1 warm-up "
                       f"({med * 1e3:.1f} ms each)")}


def reference_arm(args) -> None:
    """The reference's own CPU implementation of the path (its eager forward,
    restated in the oracle: the reference's backend never executes kernels)
    on all host threads, W warm-up and K timed steps of the same workload."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg, model, x, desc, scaling = _workload(args.workload, 0, world)
    if args.workload == "c4" and world > 1:  # the job's batch, not one rank's share
        cfg, model, x, desc, scaling = _workload(args.workload, 0, 1)
    torch.set_num_threads(os.cpu_count() or 1)
    fwd = _eager_forward(cfg, model)
    with torch.no_grad():
        # each step runs the whole batch unless K + W such forwards would exceed ~4 minutes
        xb, once = _sample_rows(fwd, x, 240.0 / max(1, args.steps + args.warmup))
        for _ in range(max(0, args.warmup - 1)):
            fwd(xb)
        ts = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            fwd(xb)
            ts.append(time.perf_counter() - t0)
    ms = 1e3 * sum(ts) / len(ts)
    tokens = xb.shape[0] * xb.shape[1]
    v = tokens / (ms / 1e3)
    job_batch = x.shape[0] * (world if args.workload == "c2" else 1)
    whole = xb.shape[0] == x.shape[0]
    sample = (f"oracle eager forward (the reference's algorithm) in {str(cfg.dtype).replace('torch.', '')}, "
              f"{'the whole workload batch' if whole else f'batch {xb.shape[0]} of {x.shape[0]}'} "
              f"({xb.shape[0]} x seq {xb.shape[1]}) per step, mean of {args.steps} steps after {args.warmup} warm-up")
    line = {"metric": "tokens/sec per forward", "value": v, "unit": "tokens/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}[cfg.dtype],
            "data": "synthetic", "config": {"workload": desc, "global_batch": job_batch, "seq_len": x.shape[1]},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c3", choices=["c1", "c2", "c3", "c4"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--timeline", type=Path, default=None, metavar="PATH",
                    help="after the timed steps, write rank 0's per-launch event timeline of one forward to PATH")
    ap.add_argument("--tp-chunks", type=int, default=4, help="c3 tensor parallel: row chunks of the all-reduce overlap")
    ap.add_argument("--tp-allreduce", choices=["auto", "multimem", "nccl"], default="auto",
                    help="c3 tensor parallel: all-reduce through NVSwitch multicast (th_allreduce) or NCCL")
    ap.add_argument("--tp-comm-sms", type=int, default=None,
                    help="c3 tensor parallel: SMs the overlapped GEMMs leave to the all-reduces (default: by rank count)")
    args = ap.parse_args()

    if args.impl == "reference":
        reference_arm(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    metric, unit = "tokens/sec per forward", "tokens/s"

    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)

    from torch_helion import CompileConfig, compile_model

    cfg, model, x, desc, scaling = _workload(args.workload, rank, world)
    tp = args.workload == "c3" and world > 1
    res = compile_model(model, (x,), CompileConfig(run_name=f"bench_{args.workload}_r{rank}", device=str(dev),
                                                   verify_passes=False, reference_check=False,
                                                   results_dir=REPO / "results", world_size=world if tp else 1,
                                                   tp_mode="heads" if tp else None, tp_chunks=args.tp_chunks,
                                                   tp_comm_sms=args.tp_comm_sms, tp_allreduce=args.tp_allreduce))
    mod = res.module
    prog = mod.program  # this rank's program (its tensor-parallel shard under TP)
    tokens = x.shape[0] * x.shape[1]
    job_tokens = tokens if tp else world * tokens  # tokens the whole job processes per step
    flushbuf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    flush = lambda: flushbuf.fill_(1.0)
    xd = x.to(dev)
    mod.load_inputs([xd])
    # one GPU / batch-sharded: the forward is replayed as one CUDA graph (the
    # per-kernel timing pass below launches the same kernels one by one);
    # tensor parallel: eager launches, the all-reduces on a second stream
    if not tp:
        mod.capture_graph()
    st = torch.cuda.current_stream()

    def barrier():
        if dist is not None:
            dist.barrier()

    mk = lambda: torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        # ---- device-resident forward
        for _ in range(max(3, args.warmup)):
            flush()
            mod.launch_all()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        ev = [(mk(), mk()) for _ in range(args.steps)]
        for e0, e1 in ev:
            flush()
            e0.record(st)
            mod.launch_all()
            e1.record(st)
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        ms = sum(a.elapsed_time(b) for a, b in ev) / args.steps
        # the same K steps again with every launch bracketed by events (on the
        # launching stream): the per-kernel times behind the roofline.  A
        # ~0.1 ms device sleep ahead of each bracket lets the host enqueue the
        # launch before the GPU reaches it, so host-side launch cost stays out
        # of the kernel's time (it does not touch memory: L2 holds what the
        # preceding kernels left, as in the real forward)
        kev = [[(mk(), mk()) for _ in mod.launches] for _ in range(args.steps)]
        for kl in kev:
            flush()
            for l, (k0, k1) in zip(mod.launches, kl):
                torch.cuda._sleep(200_000)
                k0.record(st)
                l.fn()
                k1.record(st)
        torch.cuda.synchronize()
        barrier()
        ktimes: dict[str, float] = {}
        for j, l in enumerate(mod.launches):
            ktimes[l.name] = sum(kl[j][0].elapsed_time(kl[j][1]) for kl in kev) / args.steps

        # ---- end to end through the public serving entry (CompileResult.streaming_runner):
        # every step copies its input from pinned host memory and its output back;
        # step i's copies overlap the forward of its neighbours (two slots, three
        # streams).  The L2 flush runs on the compute stream before each forward.
        xh = x.pin_memory()
        runner = res.streaming_runner(depth=2, cuda_graph=True)
        if tp:
            rows_in = runner.input_rows(xh)
            outs = [runner.output_buffer() for _ in range(2)]
            submit = lambda i: runner.submit(i, rows_in, outs[i % 2], before_forward=flush)
            h2d = rows_in.numel() * rows_in.element_size() * world   # the job's bytes (each rank its rows)
            d2h = outs[0].numel() * outs[0].element_size() * world
        else:
            outs = [runner.output_buffers() for _ in range(2)]
            submit = lambda i: runner.submit(i, [xh], outs[i % 2], before_forward=flush)
            h2d = xh.numel() * xh.element_size() * world
            d2h = outs[0][0].numel() * outs[0][0].element_size() * world
        for i in range(max(3, args.warmup)):
            submit(i)
        runner.synchronize()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = mk(), mk()
        e0.record(runner.h2d)
        for i in range(args.steps):
            submit(i)
        e1.record(runner.d2h)
        runner.synchronize()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        ms_e2e = e0.elapsed_time(e1) / args.steps
        del runner
        if args.timeline is not None:  # every rank runs it (collectives inside); rank 0 writes it
            flush()
            torch.cuda.synchronize()
            barrier()  # the ranks start the forward together
            marks = mod.timeline()
            if rank == 0:
                args.timeline.parent.mkdir(parents=True, exist_ok=True)
                args.timeline.write_text("".join(f"{t:9.3f}  {name}  rows@{r0}\n" for t, name, r0 in marks))

    # ---- per-kernel times and the dominant kernel's roofline
    peaks, peak_src = _peaks()
    top = max((l for l in mod.launches if l.kind not in ("nccl", "allreduce")), key=lambda l: ktimes[l.name])
    work = kernel_work(top, prog, mod)
    ridge = peaks["bf16_tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9)
    t_top = ktimes[top.name] / 1e3
    tensor_kind = top.kind in ("gemm", "attention") and work["flops"] / max(work["bytes"], 1) > ridge \
        and mod.dtype != torch.float32
    if tensor_kind:
        # a kernel timed inside a multi-millisecond step runs under the power cap: the sustained figure
        sustained = ms > 2.0 and "bf16_tflops_sustained" in peaks
        tc_peak = peaks["bf16_tflops_sustained"] if sustained else peaks["bf16_tflops"]
        peak_src = peak_src + (" (sustained)" if sustained else " (burst)")
        achieved, peak, ru, bound = work["flops"] / t_top / 1e12, tc_peak, "TFLOP/s", "tensor"
    else:
        achieved, peak, ru, bound = work["bytes"] / t_top / 1e9, peaks["hbm_gbs"], "GB/s", "hbm"
    traffic = None
    tf = REPO / "profiles" / f"traffic_{args.workload}{'_tp' + str(world) if tp else ''}.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get(top.name)

    ar_bytes = {l.name: l.nbytes for l in mod.launches if l.kind in ("nccl", "allreduce")}

    # ---- aggregate over ranks (max time)
    t = torch.tensor([ms, ms_e2e], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_e2e = float(t[0]), float(t[1])
    n = world
    if rank == 0:
        cb = None if (args.no_cpu_baseline or n > 1) else cpu_baseline(cfg, model, x)
        dt_name = {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}[mod.dtype]
        if tp:
            how = ("th_allreduce (NVSwitch multicast, in place on symmetric buffers)" if mod._multimem
                   else "NCCL all-reduce")
            par = (f"tp{n}: heads and FFN columns, {how} after o_proj and after down_proj, "
                   f"{args.tp_chunks} row chunks overlapping the all-reduces with the GEMMs, "
                   f"which leave {mod.tp_comm_sms} SMs to them")
            launch = f"eager launches; {'th_allreduce kernels' if mod._multimem else 'NCCL all-reduces'} on a second stream"
            entry = ("CompileResult.streaming_runner -> ShardedStreamingRunner: each rank copies its 1/N of the "
                     "rows in and out of pinned host memory, NCCL all-gather of the input rows, tensor-parallel "
                     "forward; copies overlapped with neighbouring forwards")
        else:
            par = (f"dp{n}: batch-sharded, no communication" if n > 1 else "single GPU")
            launch = "one CUDA graph per forward"
            entry = ("CompileResult.streaming_runner -> StreamingRunner: 2 slots, CUDA-graph forward, "
                     "H2D / compute / D2H streams")
        line = {
            "metric": metric, "value": job_tokens / (ms / 1e3), "unit": unit, "n_gpus": n, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": dt_name, "data": "synthetic (seeded N(0,1) inputs, N(0,0.02) weights, BASELINE shapes)",
            "config": {"workload": desc, "global_batch": x.shape[0] if tp else n * x.shape[0], "seq_len": x.shape[1],
                       "parallelism": par, "l2": "flushed between steps (256 MiB write, untimed)",
                       "kernels_per_forward": mod.n_launches, "launch": launch},
            "roofline": {"bound": bound, "kernel": f"{top.name} ({top.kind})", "achieved": achieved, "peak": peak,
                         "unit": ru, "frac": achieved / peak, "peak_source": peak_src,
                         "algorithmic_bytes": work["bytes"], "algorithmic_flops": work["flops"],
                         "launch_ms": ktimes[top.name], "traffic": traffic},
            "e2e": {"value": job_tokens / (ms_e2e / 1e3), "unit": unit, "ms_per_step": ms_e2e, "entry": entry,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    # the larger copy's bytes per GPU per e2e step time: the host link rate sustained
                    "copy_gbs_per_gpu": max(h2d, d2h) / n / ms_e2e / 1e6,
                    "bound": "host copies" if ms_e2e > 1.2 * ms else "device forward"},
            "gpu_launches": mod.n_launches * args.steps,
            "clocks": clocks.summary(),
            "kernels_ms": ktimes,
            "cpu_baseline": cb,
        }
        if tp:
            # each all-reduce on its own: the bytes it sums over the time it took (algorithm bandwidth)
            line["collectives"] = {
                l.name: {"kind": "th_allreduce (NVSwitch multicast)" if l.kind == "allreduce" else "NCCL all_reduce",
                         "bytes": ar_bytes[l.name], "ms": ktimes[l.name],
                         "algbw_gbs": ar_bytes[l.name] / ktimes[l.name] / 1e6}
                for l in mod.launches if l.kind in ("nccl", "allreduce")}
        if dist is not None:
            line["nccl"] = {"backend": dist.get_backend(), "ranks": dist.get_world_size(),
                            "tp_allreduce": "multimem" if getattr(mod, "_multimem", False) else "nccl",
                            "nvls_env": os.environ.get("NCCL_NVLS_ENABLE", "unset (NCCL default)"),
                            "nccl_version": ".".join(map(str, torch.cuda.nccl.version()))}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
