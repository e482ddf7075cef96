"""Execute an OpIR Program on a B200 through the C ABI.

The B200 twin of the reference interpreter (src/torch_helion/codegen/
interpret.py:54-65, ``run_program``): it walks ``program.kernels`` in order
and launches each one -- but on the GPU, through ``libth_b200.so``.
Everything is prepared once in :class:`CompiledProgram`:

* parameters are uploaded in the layout the kernels want (GEMM weights
  transposed to [N, K] and concatenated per kernel, SwiGLU gate/up
  interleaved in 64-row blocks, rope/conv/scan constants in fp32);
* every intermediate gets a device buffer; a GEMM's sibling outputs are
  column views of one buffer, its fp32 tail (the scan's dt) a second one;
* the RMSNorm row statistics come from the cheapest producer: the
  ``ss_out`` partials of the GEMM that wrote the tensor, the scan's
  per-head ``gss``, or a ``th_rowstat`` launch;
* each kernel becomes a closure with fixed pointers, so the whole forward
  can also be captured in one CUDA graph.

There is no CPU fallback: without a CUDA device or the built library this
raises :class:`~torch_helion.b200.lib.B200KernelError`.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Sequence

import torch

from ..optimizer.opir import KernelArg, Program
from . import lib
from .lower import GemmPlan, MacroPlan, fp32_outputs, lower_gemm, lower_macro

# launch kinds that exchange data between the ranks (run on the communication stream when chunked)
_COLLECTIVES = ("nccl", "allreduce")
_TORCH_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16, "int64": torch.int64}


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


@dataclass
class KernelLaunch:
    name: str
    kind: str
    fn: Callable[[], None]
    # the same launch restricted to rows [r0, r1) of every row-indexed operand
    # (None: the kernel does not decompose by rows, e.g. attention or RoPE)
    fn_rows: Callable[[int, int], None] | None = None
    # bytes a collective sums per call (0 for compute kernels)
    nbytes: int = 0


def _chunk_bounds(rows: int, n: int) -> list[tuple[int, int]]:
    """Row ranges of the ``n`` chunks of the tensor-parallel tail, multiples of 128 rows.

    With three or more chunks the first and the last are half as tall as the
    rest: the first chunk's all-reduce is the one the compute stream can wait
    for (only the next chunk's o_proj runs beside it), and the last chunk's
    all-reduce ends the forward with nothing to hide behind."""
    w = [0.5] + [1.0] * (n - 2) + [0.5] if n >= 3 else [1.0] * n
    tiles = (rows + 127) // 128
    edges, acc = [0], 0.0
    for i, wi in enumerate(w[:-1]):
        acc += wi
        e = int(round(acc / sum(w) * tiles))
        edges.append(min(max(e, edges[-1] + 1), tiles - (n - 1 - i)))
    edges.append(tiles)
    return [(a * 128, min(rows, b * 128)) for a, b in zip(edges, edges[1:])]


class CompiledProgram:
    """A Program bound to device memory on one GPU."""

    def __init__(self, program: Program, params: dict[str, torch.Tensor], device: str | torch.device = "cuda",
                 tp_rank: int = 0, tp_world: int = 1, allreduce: Callable[[torch.Tensor], None] | None = None,
                 shared_params: dict | None = None, tp_chunks: int = 4, tp_comm_sms: int | None = None,
                 tp_allreduce: str = "auto") -> None:
        if not torch.cuda.is_available():
            raise lib.B200KernelError("CompiledProgram needs a CUDA device (there is no CPU fallback)")
        lib.load()
        self.program = program
        self.device = torch.device(device)
        self.dtype = _TORCH_DTYPES[program.metadata.get("dtype", "float32")]
        self.params = params
        self.views: dict[str, torch.Tensor] = {}
        self.launches: list[KernelLaunch] = []
        # device copies of the parameters, keyed by layout; a second program of
        # the same Program (another pipeline slot) passes the first one's dict
        self._dev_params: dict[tuple, torch.Tensor] = shared_params if shared_params is not None else {}
        self._graph: torch.cuda.CUDAGraph | None = None
        self._ssd_ws: torch.Tensor | None = None
        self.tp_rank, self.tp_world, self.allreduce = tp_rank, tp_world, allreduce
        self.tp_chunks = tp_chunks
        if tp_allreduce not in ("auto", "multimem", "nccl"):
            raise ValueError(f"tp_allreduce must be auto, multimem or nccl, not {tp_allreduce!r}")
        # Measured on B200 (C3 block, 4 chunks): the multicast kernel on 16 SMs of its own overlaps the
        # GEMMs best -- 8 ranks: 2.52 ms per forward against 2.69 with 24 SMs and 3.14 over NCCL; 2 ranks
        # (with the row statistics folded into it): 6.64 ms against 7.21 over NCCL with every SM to the
        # GEMMs.  Where multicast is missing, NCCL runs with every SM left to the GEMMs.
        self.tp_allreduce = tp_allreduce
        # SMs left to the collectives while the chunked schedule overlaps them with GEMMs: the GEMMs'
        # persistent grids are capped at (SMs - tp_comm_sms) there, and th_allreduce runs on that many CTAs
        self._comm_sms_arg = tp_comm_sms
        self.tp_comm_sms = tp_comm_sms if tp_comm_sms is not None else 16
        self._gemm_sm_limit = 0  # read by every GEMM launch when it runs
        self._multimem = False  # all-reduces through th_allreduce on symmetric buffers (decided in _build)
        self._symmetric: list = []
        self._sym_views: dict = {}  # tensor name -> the SymmetricRows whose whole row it is
        self._pipe: tuple | None = None  # chunked tensor-parallel schedule (see _plan_tp_pipeline)
        with torch.cuda.device(self.device):
            self._build()
            self._plan_tp_pipeline()

    # ------------------------------------------------------------ parameters
    def _param(self, name: str, kind: str = "raw", dtype: torch.dtype | None = None) -> torch.Tensor:
        key = (name, kind, dtype)
        if key not in self._dev_params:
            v = self.params[name]
            if kind == "f32vec":
                v = v.float().reshape(-1)
            elif kind == "f32":
                v = v.float()
            t = v.to(device=self.device, dtype=dtype or v.dtype).contiguous()
            self._dev_params[key] = t
        return self._dev_params[key]

    def _gemm_weight(self, plan: GemmPlan, n_main_pad: int, n_tail_pad: int) -> torch.Tensor:
        """[N_total, K] weight in the column order of the plan (rows padded)."""
        key = ("gemm_w", tuple(s.rhs for s in plan.segments), n_main_pad, n_tail_pad)
        if key in self._dev_params:
            return self._dev_params[key]
        K = plan.k
        dt = self.dtype
        if plan.swiglu is not None:
            from ..optimizer.param_transforms import swiglu_interleave

            wg = self.params[plan.swiglu[0]].t().float()
            wu = self.params[plan.swiglu[1]].t().float()
            w = swiglu_interleave(wg, wu).to(dt)
        else:
            main = [self.params[s.rhs].t().float() for s in plan.segments if s.kind != "tail"]
            tail = [self.params[s.rhs].t().float() for s in plan.segments if s.kind == "tail"]
            rows = []
            m = torch.cat(main, 0) if main else torch.zeros(0, K)
            rows.append(m)
            if n_main_pad > m.shape[0]:
                rows.append(torch.zeros(n_main_pad - m.shape[0], K))
            if tail:
                t = torch.cat(tail, 0)
                rows.append(t)
                if n_tail_pad > t.shape[0]:
                    rows.append(torch.zeros(n_tail_pad - t.shape[0], K))
            w = torch.cat(rows, 0).to(dt)
        w = w.to(self.device).contiguous()
        self._dev_params[key] = w
        return w

    # --------------------------------------------------------------- buffers
    def _empty(self, rows: int, cols: int, dtype: torch.dtype) -> torch.Tensor:
        return torch.empty(rows, cols, device=self.device, dtype=dtype)

    def _view(self, arg: KernelArg) -> torch.Tensor:
        if arg.tensor in self.program.params:
            raise lib.B200KernelError(f"{arg.tensor} is a constant, not an activation")
        v = self.views[arg.tensor]
        return v[:, arg.cols[0]:arg.cols[1]] if arg.cols else v

    def _build(self) -> None:
        prog = self.program
        T_of = lambda name: prog.tensors[name].shape[0]
        for name in prog.inputs:
            t = prog.tensors[name]
            dt = _TORCH_DTYPES[t.dtype]
            cols = t.shape[1] if dt == torch.int64 else _round_up(t.shape[1], 8)
            buf = self._empty(t.shape[0], cols, dt)
            self.views[name] = buf if dt == torch.int64 else buf[:, : t.shape[1]]
        if self.tp_world > 1 and self.tp_allreduce != "nccl" and any(self._allreduced(k) for k in prog.kernels):
            import torch.distributed as dist

            from .collectives import multimem_available

            # only over a process group of this program's ranks; otherwise the caller's all-reduce
            # (e.g. a stand-in that runs one rank's shard alone) is used
            grouped = dist.is_available() and dist.is_initialized() and dist.get_world_size() == self.tp_world
            self._multimem = grouped and multimem_available(self.device)  # the same answer on every rank
            if not self._multimem and self.tp_allreduce == "multimem":
                raise lib.B200KernelError("tp_allreduce='multimem' but this node has no multicast symmetric memory")
        if not self._multimem and self._comm_sms_arg is None:
            self.tp_comm_sms = 0  # NCCL beside GEMMs on every SM measured best without the multicast kernel
        f32 = fp32_outputs(prog)
        plans = {}
        for spec in prog.kernels:
            plans[spec.name] = lower_gemm(spec, prog.tensors, f32) if spec.kind == "gemm" else lower_macro(spec, prog.tensors)
        # who computes the row statistics of each GEMM LHS
        need_ss = {next(a.tensor for a in s.args if a.role == "lhs") for s in prog.kernels if s.kind == "gemm" and s.sumsq}
        self._ss_parts: dict[str, torch.Tensor] = {}
        ss_by_producer: dict[str, str] = {}
        for tname in need_ss:
            prod = prog.producer(tname)
            if prod is None:
                continue
            p = plans[prod.name]
            if isinstance(p, GemmPlan) and p.outputs.get(tname, (None,))[0] == "main" and p.outputs[tname][1] == 0 \
                    and p.outputs[tname][2] == p.n_main and not self._allreduced(prod):
                ss_by_producer[tname] = prod.name
            elif isinstance(p, MacroPlan) and p.kind == "ssd" and p.attrs.get("gate"):
                ss_by_producer[tname] = prod.name
        for spec in prog.kernels:
            p = plans[spec.name]
            if isinstance(p, GemmPlan):
                self._add_gemm(spec.name, spec, p, need_ss, ss_by_producer)
            else:
                self._add_macro(spec.name, p, need_ss, ss_by_producer)
        self.outputs = list(prog.outputs)

    def _allreduced(self, spec) -> bool:
        return self.tp_world > 1 and spec.attrs.get("tp_allreduce", False)

    def _row_parts(self, tname: str, ss_by_producer: dict[str, str]) -> torch.Tensor:
        """fp32 [T, nparts] whose row sums are sum(x^2) of tensor ``tname``."""
        if tname in self._ss_parts:
            return self._ss_parts[tname]
        sym = self._sym_views.get(tname)
        if sym is not None and sym.world > 1 and 128 % sym.world == 0 and sym.buf.shape[0] % 128 == 0:
            # the multicast all-reduce that produces the tensor stores each row's sum of squares
            # (every chunk is whole 128-row tiles, so every rank's slice of a chunk is whole rows)
            sym.stats = True
            self._ss_parts[tname] = sym.sumsq.view(-1, 1)
            return self._ss_parts[tname]
        # no producer writes it: a th_rowstat launch right before the consumer
        x = self.views[tname]
        parts = self._empty(x.shape[0], 1, torch.float32)
        self.launches.append(KernelLaunch(
            f"rowstat({tname})", "rowstat", lambda x=x, parts=parts: lib.rowstat(x, parts.view(-1)),
            lambda r0, r1, x=x, parts=parts: lib.rowstat(x[r0:r1], parts.view(-1)[r0:r1])))
        self._ss_parts[tname] = parts
        return parts

    def _add_gemm(self, kname: str, spec, p: GemmPlan, need_ss, ss_by_producer) -> None:
        T = p.rows
        n_main_pad = _round_up(p.n_main, 8)
        n_tail = p.n_tail
        n_tail_pad = _round_up(n_tail, 8) if n_tail else 0
        W = self._gemm_weight(p, n_main_pad, n_tail_pad)
        sym = None
        if self._multimem and self._allreduced(spec):  # reduced in place through NVSwitch multicast
            from .collectives import SymmetricRows

            sym = SymmetricRows(T, max(n_main_pad, 8), self.dtype, self.device,
                                ctas=self.tp_comm_sms if self.tp_comm_sms > 0 else 16)
            self._symmetric.append(sym)
            out = sym.buf
        else:
            out = self._empty(T, max(n_main_pad, 8), self.dtype)
        tail = self._empty(T, n_tail_pad, torch.float32) if n_tail else None
        for tname, (where, c0, c1) in p.outputs.items():
            self.views[tname] = (out if where == "main" else tail)[:, c0:c1]
            if sym is not None and where == "main" and c0 == 0 and c1 == out.shape[1]:
                self._sym_views[tname] = sym
        lhs = self._view(p.lhs)
        kw: dict = {}
        if p.rowscale is not None:
            kw.update(rs_parts=self._row_parts(p.lhs.tensor, ss_by_producer), rs_inv_k=p.rowscale[0], rs_eps=p.rowscale[1])
        # activation segment (acc column space == output column space without SwiGLU)
        col = 0
        for s in p.segments:
            if s.kind == "act":
                kw.update(act=lib.ACT_CODES[p.act], act_begin=col, act_end=col + s.width)
            if s.kind != "tail":
                col += s.width
        if n_tail:
            act_code = lib.ACT_CODES[p.act]
            kw.update(act=act_code, act_begin=n_main_pad, act_end=n_main_pad + n_tail, out2=tail, tail_begin=n_main_pad)
        if p.bias is not None:
            kw["bias"] = self._param(p.bias, "f32vec", torch.float32)
        if p.rope is not None:
            r0 = sum(s.width for s in p.segments if s.kind == "rope")
            kw.update(rope_cos=self._param(p.rope[0], "f32", torch.float32),
                      rope_sin=self._param(p.rope[1], "f32", torch.float32), rope_begin=0, rope_end=r0,
                      rope_head_dim=p.rope[2])
        if p.swiglu is not None:
            kw["swiglu"] = True
        if p.residual is not None:
            kw["residual"] = self._view(p.residual)
        # row statistics for a consumer, from this kernel's epilogue
        for tname, prod in ss_by_producer.items():
            if prod == kname:
                parts = self._empty(T, (n_main_pad + 63) // 64, torch.float32)
                self._ss_parts[tname] = parts
                kw["ss_out"] = parts
        d = out if n_tail == 0 or n_main_pad == 0 else out[:, :n_main_pad]  # all-tail GEMMs write no main output
        fn_rows = None
        if p.rope is None:  # RoPE positions follow the row index: no row slicing
            row_kw = [k for k in ("rs_parts", "residual", "out2", "ss_out") if k in kw]

            def fn_rows(r0, r1, lhs=lhs, W=W, d=d, kw=kw, row_kw=row_kw):
                kr = dict(kw)
                for k in row_kw:
                    kr[k] = kw[k][r0:r1]
                lib.gemm(lhs[r0:r1], W, d[r0:r1], sm_limit=self._gemm_sm_limit, **kr)
        self.launches.append(KernelLaunch(kname, "gemm", lambda lhs=lhs, W=W, d=d, kw=kw: lib.gemm(
            lhs, W, d, sm_limit=self._gemm_sm_limit, **kw),
                                          fn_rows))
        if sym is not None:
            self.launches.append(KernelLaunch(f"allreduce({kname})", "allreduce",
                                              lambda sym=sym, T=T: sym.allreduce_rows(0, T), sym.allreduce_rows,
                                              nbytes=T * sym.row_bytes))
        elif self._allreduced(spec):
            buf = out  # the whole (contiguous) buffer; zero-weight pad columns sum to zero
            self.launches.append(KernelLaunch(f"allreduce({kname})", "nccl", lambda buf=buf: self.allreduce(buf),
                                              lambda r0, r1, buf=buf: self.allreduce(buf[r0:r1]),
                                              nbytes=buf.numel() * buf.element_size()))

    def _add_macro(self, kname: str, p: MacroPlan, need_ss, ss_by_producer) -> None:
        prog = self.program
        a = p.attrs
        out_t = prog.tensors[p.output]
        T, C = out_t.shape
        out = self._empty(T, _round_up(C, 8), self.dtype)[:, :C]
        self.views[p.output] = out
        A = p.args
        if p.kind == "attention":
            q, k, v = self._view(A["q"]), self._view(A["k"]), self._view(A["v"])
            fn = lambda: lib.attention(q, k, v, out, batch=a["batch"], seq=a["seq"], hq=a["heads"],
                                       hkv=a.get("kv_heads", a["heads"]), head_dim=a["head_dim"], scale=a["scale"],
                                       causal=bool(a.get("causal")))
        elif p.kind == "causal_conv1d":
            x = self._view(A["x"])
            w = self._param(A["w"].tensor, "f32", torch.float32)
            act = lib.ACT_SILU if a.get("act") == "silu" else lib.ACT_NONE
            fn = lambda: lib.conv1d(x, w, out, batch=a["batch"], seq=a["seq"], act=act)
        elif p.kind == "rmsnorm":
            x = self._view(A["x"])
            gain = self._param(A["gain"].tensor, "f32vec", torch.float32)
            fn = lambda: lib.rmsnorm(x, gain, a["eps"], out=out)
        elif p.kind == "embedding":
            ids = self.views[A["ids"].tensor].reshape(-1)
            table = self._param(A["table"].tensor, "raw", self.dtype)
            fn = lambda: lib.embedding(ids, table, out)
        elif p.kind == "ssd":
            x, dt, B, C_ = self._view(A["x"]), self._view(A["dt"]), self._view(A["B"]), self._view(A["C"])
            if dt.dtype != torch.float32:
                raise lib.B200KernelError(f"{kname}: dt must be fp32")
            Av = self._param(A["A"].tensor, "f32vec", torch.float32)
            Dv = self._param(A["D"].tensor, "f32vec", torch.float32) if "D" in A else None
            z = self._view(A["z"]) if "z" in A else None
            chunk = 256 if a["seq"] >= 256 else _round_up(a["seq"], 64)
            need = lib.ssd_workspace_size(a["batch"], a["seq"], a["heads"], a["head_dim"], a["state_dim"], chunk)
            if self._ssd_ws is None or self._ssd_ws.numel() < need:
                self._ssd_ws = torch.empty(need, dtype=torch.uint8, device=self.device)
            ws = self._ssd_ws
            gss = None
            if ss_by_producer.get(p.output) == kname:
                gss = self._empty(T, a["heads"], torch.float32)
                self._ss_parts[p.output] = gss
            fn = lambda: lib.ssd(x, dt, Av, B, C_, out, batch=a["batch"], seq=a["seq"], heads=a["heads"],
                                 head_dim=a["head_dim"], ngroups=a["ngroups"], state_dim=a["state_dim"], chunk=chunk,
                                 D=Dv, z=z, gss=gss, workspace=ws)
        else:
            raise lib.B200KernelError(f"{kname}: unknown kind {p.kind}")
        self.launches.append(KernelLaunch(kname, p.kind, fn))

    # ------------------------------------------------------------------ run
    def load_inputs(self, inputs: Sequence[torch.Tensor]) -> None:
        if len(inputs) != len(self.program.inputs):
            raise ValueError(f"expected {len(self.program.inputs)} inputs, got {len(inputs)}")
        for name, x in zip(self.program.inputs, inputs):
            dst = self.views[name]
            src = x.reshape(dst.shape) if dst.dim() == 1 else x.reshape(dst.shape[0], -1)
            dst.copy_(src, non_blocking=True)

    def _plan_tp_pipeline(self) -> None:
        """Row-chunked schedule of the tensor-parallel tail of the program.

        From the GEMM whose output is the first all-reduce to the end (o_proj,
        all-reduce, row statistics, gate|up, down, all-reduce in the Llama
        block) every launch works row by row, so the rows are cut into chunks:
        chunk c's all-reduce runs on a communication stream while chunk c+1's
        GEMMs run on the compute stream, and the part after the first all-reduce
        of chunk c waits only for that chunk's all-reduce.  The rows of every
        chunk are a multiple of 128 (whole GEMM row tiles); the first and the
        last chunk are half as tall as the others (see ``_chunk_bounds``)."""
        if self.tp_world <= 1 or self.tp_chunks <= 1:
            return
        first = next((i for i, l in enumerate(self.launches) if l.kind in _COLLECTIVES), None)
        if first is None or first == 0:
            return
        seg = self.launches[first - 1:]
        if any(l.fn_rows is None for l in seg):
            return
        rows = {v.shape[0] for v in self.views.values() if v.dim() == 2}
        T = max(rows)
        n = min(self.tp_chunks, T // 128)
        if n <= 1:
            return
        bounds = _chunk_bounds(T, n)
        pre = seg[:2]    # the GEMM and its all-reduce
        post = seg[2:]   # everything after, per chunk
        self._pipe = (self.launches[:first - 1], pre, post, bounds, torch.cuda.Stream(device=self.device))

    def _launch_pipelined(self) -> None:
        prefix, pre, post, bounds, comm = self._pipe
        main = torch.cuda.current_stream()
        for l in prefix:
            l.fn()
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        self._gemm_sm_limit = max(2, sms - self.tp_comm_sms) if self.tp_comm_sms > 0 else 0
        try:
            self._run_chunks(pre, post, bounds, comm, main)
        finally:
            self._gemm_sm_limit = 0

    def _run_chunks(self, pre, post, bounds, comm, main) -> None:

        def collective(l, r0, r1) -> torch.cuda.Event:
            ready = torch.cuda.Event()
            ready.record(main)
            comm.wait_event(ready)
            with torch.cuda.stream(comm):
                l.fn_rows(r0, r1)
            done = torch.cuda.Event()
            done.record(comm)
            return done

        def run(chunk, r0, r1) -> torch.cuda.Event | None:
            last = None
            for l in chunk:
                if l.kind in _COLLECTIVES:
                    last = collective(l, r0, r1)
                else:
                    if last is not None:  # compute after a collective of the same rows
                        main.wait_event(last)
                        last = None
                    l.fn_rows(r0, r1)
            return last

        pending = [run(pre, *bounds[0])]
        tail = None
        for c, (r0, r1) in enumerate(bounds):
            if c + 1 < len(bounds):
                pending.append(run(pre, *bounds[c + 1]))
            if pending[c] is not None:
                main.wait_event(pending[c])
            tail = run(post, r0, r1) or tail
        if tail is not None:
            main.wait_event(tail)  # every chunk's last collective precedes it on the comm stream

    def launch_all(self) -> None:
        if self._graph is not None:
            self._graph.replay()
            return
        if self._pipe is not None:
            self._launch_pipelined()
            return
        for l in self.launches:
            l.fn()

    def timeline(self) -> list[tuple[float, str, int]]:
        """One eager forward with a CUDA event recorded after every launch on the stream it went to:
        [(ms from the forward's start to the launch's end, launch name, first row or -1)], sorted by
        time.  Under tensor parallelism every rank must call it (the collectives run inside)."""
        marks: list[tuple[str, int, torch.cuda.Event]] = []
        saved = [(l, l.fn, l.fn_rows) for l in self.launches]

        def mark(name: str, r0: int) -> None:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            marks.append((name, r0, e))

        for l, fn, fr in saved:
            l.fn = lambda fn=fn, name=l.name: (fn(), mark(name, -1))
            if fr is not None:
                l.fn_rows = lambda r0, r1, fr=fr, name=l.name: (fr(r0, r1), mark(name, r0))
        graph, self._graph = self._graph, None
        try:
            with torch.cuda.device(self.device):
                torch.cuda.synchronize()
                start = torch.cuda.Event(enable_timing=True)
                start.record()
                self.launch_all()
                torch.cuda.synchronize()
        finally:
            self._graph = graph
            for l, fn, fr in saved:
                l.fn, l.fn_rows = fn, fr
        return sorted((start.elapsed_time(e), name, r0) for name, r0, e in marks)

    def output_views(self) -> list[torch.Tensor]:
        shapes = self.program.metadata.get("output_shapes", {})
        outs = []
        for o in self.outputs:
            v = self.views[o]
            outs.append(v.reshape(shapes[o]) if o in shapes and v.is_contiguous() else
                        (v.contiguous().reshape(shapes[o]) if o in shapes else v))
        return outs

    def __call__(self, *inputs: torch.Tensor) -> list[torch.Tensor]:
        with torch.cuda.device(self.device):
            self.load_inputs(inputs)
            self.launch_all()
            return self.output_views()

    def capture_graph(self) -> None:
        """Record every launch of the forward into one CUDA graph (after one
        eager run, so one-time host set-up stays out of the capture)."""
        with torch.cuda.device(self.device):
            for l in self.launches:
                l.fn()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for l in self.launches:
                    l.fn()
            self._graph = g

    @property
    def n_launches(self) -> int:
        """Kernels of this library launched per forward (NCCL's own kernels excluded)."""
        if self._pipe is not None:
            prefix, pre, post, bounds, _ = self._pipe
            per_chunk = sum(1 for l in pre + post if l.kind != "nccl")
            return sum(1 for l in prefix if l.kind != "nccl") + len(bounds) * per_chunk
        return sum(1 for l in self.launches if l.kind != "nccl")

    def launch_names(self) -> list[str]:
        return [l.name for l in self.launches]


class StreamingRunner:
    """Serve a stream of batches from pinned host memory.

    ``depth`` copies of the program (one set of activation buffers each, the
    weights shared) rotate over three CUDA streams: the host->device copy of
    batch i+1 (one copy engine) and the device->host copy of batch i-1 (the
    other) run while the SMs compute batch i.  Events order every reuse of a
    slot: its inputs are overwritten only after its previous forward, its
    outputs only after their previous copy-out.  Steady-state time per batch is
    max(forward, H2D, D2H) instead of their sum.
    """

    def __init__(self, program: Program, params: dict[str, torch.Tensor], device: str | torch.device = "cuda",
                 depth: int = 2, cuda_graph: bool = False) -> None:
        if depth < 1:
            raise ValueError("depth must be >= 1")
        first = CompiledProgram(program, params, device)
        self.slots = [first] + [CompiledProgram(program, params, device, shared_params=first._dev_params)
                                for _ in range(depth - 1)]
        self.device = first.device
        with torch.cuda.device(self.device):
            if cuda_graph:
                for s in self.slots:
                    s.capture_graph()
            self.h2d, self.compute, self.d2h = (torch.cuda.Stream(self.device) for _ in range(3))
            ev = lambda: [torch.cuda.Event() for _ in self.slots]
            self._loaded, self._computed, self._drained = ev(), ev(), ev()
        self._used = [False] * depth

    def output_buffers(self, pin: bool = True) -> list[torch.Tensor]:
        """Host tensors shaped like one batch's outputs (pinned)."""
        return [torch.empty(v.shape, dtype=v.dtype, pin_memory=pin) for v in self.slots[0].output_views()]

    def submit(self, i: int, inputs: Sequence[torch.Tensor], outputs: Sequence[torch.Tensor],
               before_forward: Callable[[], None] | None = None) -> None:
        """Enqueue batch ``i`` (host ``inputs`` -> host ``outputs``); returns at once."""
        k = i % len(self.slots)
        s = self.slots[k]
        with torch.cuda.device(self.device):
            if self._used[k]:
                self.h2d.wait_event(self._computed[k])
            with torch.cuda.stream(self.h2d):
                s.load_inputs(inputs)
                self._loaded[k].record(self.h2d)
            self.compute.wait_event(self._loaded[k])
            if self._used[k]:
                self.compute.wait_event(self._drained[k])
            with torch.cuda.stream(self.compute):
                if before_forward is not None:
                    before_forward()
                s.launch_all()
                self._computed[k].record(self.compute)
            self.d2h.wait_event(self._computed[k])
            with torch.cuda.stream(self.d2h):
                for o, v in zip(outputs, s.output_views()):
                    o.copy_(v.reshape(o.shape), non_blocking=True)
                self._drained[k].record(self.d2h)
        self._used[k] = True

    def run(self, batches: Sequence[Sequence[torch.Tensor]], outputs: Sequence[Sequence[torch.Tensor]]) -> None:
        """Serve every batch and wait for the last copy-out."""
        for i, (inp, out) in enumerate(zip(batches, outputs)):
            self.submit(i, inp, out)
        self.synchronize()

    def synchronize(self) -> None:
        self.d2h.synchronize()

    @property
    def n_launches(self) -> int:
        return self.slots[0].n_launches


class ShardedStreamingRunner:
    """Serve a stream of batches on a tensor-parallel group (one process per
    GPU) with the host I/O sharded by rows.

    Every rank owns rows ``[rank*T/world, (rank+1)*T/world)`` of each batch
    (T = batch * seq tokens): it copies only those rows in from pinned host
    memory, the ranks all-gather the rows over NVLink (NCCL) into the
    program's input, every rank runs its head/column shard of the forward
    (with its all-reduces), and each rank copies only its own rows of the
    (replicated) output back.  The host link carries 1/world of the batch per
    GPU instead of all of it.

    Two device staging slots rotate over three streams: the copy-in of batch
    i+1 and the copy-out of batch i-1 run while batch i computes; events order
    every reuse of a slot."""

    def __init__(self, module: "CompiledProgram", depth: int = 2) -> None:
        import torch.distributed as dist

        if module.tp_world <= 1:
            raise ValueError("ShardedStreamingRunner needs a tensor-parallel module (world_size > 1)")
        if len(module.program.inputs) != 1 or len(module.outputs) != 1:
            raise ValueError("ShardedStreamingRunner serves programs with one input and one output")
        self.m, self.dist = module, dist
        self.rank, self.world = module.tp_rank, module.tp_world
        self.device = module.device
        xin = module.views[module.program.inputs[0]]
        yout = module.views[module.outputs[0]]
        T = xin.shape[0]
        if T % self.world or not xin.is_contiguous() or yout.shape[0] != T:
            raise ValueError(f"{T} rows do not split evenly over {self.world} ranks (or the input is strided)")
        self.T, self.rows = T, T // self.world
        self.r0 = self.rank * self.rows
        self.xin, self.yout = xin, yout
        with torch.cuda.device(self.device):
            self.x_stage = [torch.empty((self.rows,) + tuple(xin.shape[1:]), dtype=xin.dtype, device=self.device)
                            for _ in range(depth)]
            self.y_stage = [torch.empty((self.rows,) + tuple(yout.shape[1:]), dtype=yout.dtype, device=self.device)
                            for _ in range(depth)]
            self.h2d, self.compute, self.d2h = (torch.cuda.Stream(self.device) for _ in range(3))
            ev = lambda: [torch.cuda.Event() for _ in range(depth)]
            self._loaded, self._gathered, self._computed, self._drained = ev(), ev(), ev(), ev()
        self._used = [False] * depth

    def input_rows(self, batch: torch.Tensor) -> torch.Tensor:
        """This rank's rows of a full host batch (a view, no copy)."""
        return batch.reshape(self.T, -1)[self.r0:self.r0 + self.rows]

    def output_buffer(self, pin: bool = True) -> torch.Tensor:
        """A host tensor for this rank's rows of one batch's output."""
        return torch.empty(tuple(self.y_stage[0].shape), dtype=self.yout.dtype, pin_memory=pin)

    def submit(self, i: int, rows_in: torch.Tensor, rows_out: torch.Tensor,
               before_forward: Callable[[], None] | None = None) -> None:
        """Enqueue batch ``i``: ``rows_in`` (host, this rank's rows) -> ``rows_out`` (host); returns at once.
        Every rank must submit the same sequence of batches (the all-gather is collective)."""
        k = i % len(self.x_stage)
        with torch.cuda.device(self.device):
            if self._used[k]:
                self.h2d.wait_event(self._gathered[k])
            with torch.cuda.stream(self.h2d):
                self.x_stage[k].copy_(rows_in.reshape(self.x_stage[k].shape), non_blocking=True)
                self._loaded[k].record(self.h2d)
            self.compute.wait_event(self._loaded[k])
            if self._used[k]:
                self.compute.wait_event(self._drained[k])
            with torch.cuda.stream(self.compute):
                self.dist.all_gather_into_tensor(self.xin.view(self.world, *self.x_stage[k].shape), self.x_stage[k])
                self._gathered[k].record(self.compute)
                if before_forward is not None:
                    before_forward()
                self.m.launch_all()
                self.y_stage[k].copy_(self.yout[self.r0:self.r0 + self.rows])
                self._computed[k].record(self.compute)
            self.d2h.wait_event(self._computed[k])
            with torch.cuda.stream(self.d2h):
                rows_out.copy_(self.y_stage[k].reshape(rows_out.shape), non_blocking=True)
                self._drained[k].record(self.d2h)
        self._used[k] = True

    def synchronize(self) -> None:
        self.d2h.synchronize()

    @property
    def n_launches(self) -> int:
        return self.m.n_launches


def run_program(program: Program, params: dict[str, torch.Tensor], inputs, device="cuda") -> dict[str, torch.Tensor]:
    """Reference-shaped entry (interpret.py:54-65): run all kernels, return
    the produced tensors by name (device tensors)."""
    cp = CompiledProgram(program, params, device)
    if isinstance(inputs, dict):
        inputs = [inputs[n] for n in program.inputs]
    cp(*inputs)
    return dict(cp.views)


def program_outputs(program: Program, params: dict[str, torch.Tensor], inputs, device="cuda") -> list[torch.Tensor]:
    cp = CompiledProgram(program, params, device)
    if isinstance(inputs, dict):
        inputs = [inputs[n] for n in program.inputs]
    return [o.clone() for o in cp(*inputs)]


__all__ = ["CompiledProgram", "KernelLaunch", "StreamingRunner", "ShardedStreamingRunner", "run_program", "program_outputs", "math"]
