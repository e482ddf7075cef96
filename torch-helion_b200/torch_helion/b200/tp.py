"""Tensor parallelism of a Program over attention heads and FFN columns.

The reference has no parallelism (its only "parallel" notion is the spatial
grid of one Loom kernel).  On a B200 node the Llama block is split the
Megatron way across ``world`` GPUs, one process per GPU:

* GEMM kernels producing the attention's q/k/v become column-parallel:
  every segment keeps its rank's block of heads (RoPE is per head, so the
  epilogue is unchanged); the attention kernel runs heads/world query heads
  and kv_heads/world KV heads;
* a SwiGLU GEMM kernel (gate|up) keeps its rank's 1/world of the FFN columns;
* GEMM kernels whose LHS is one of those sharded tensors (o_proj, down_proj)
  become row-parallel: each rank multiplies its K-slice, only rank 0 adds the
  residual, and the kernel is marked ``tp_allreduce`` -- the runtime sums the
  partial outputs with one NCCL all-reduce over NVLink right after it.
Everything else (norm statistics, the residual stream) stays replicated.
A program that does not decompose this way raises :class:`TPError`.
"""

from __future__ import annotations

import copy

import torch

from ..capture.opgraph import TensorType
from ..optimizer.opir import Program


class TPError(RuntimeError):
    pass


def _acc_of_output(spec, value: str) -> set[str]:
    """Accumulators an epilogue value depends on."""
    ops = {o.name: o for o in spec.epilogue}
    accs = {g.acc for g in spec.gemms}
    seen, stack, out = set(), [value], set()
    while stack:
        v = stack.pop()
        if v in seen:
            continue
        seen.add(v)
        if v in accs:
            out.add(v)
        elif v in ops:
            stack.extend(ops[v].inputs)
    return out


def shard_program(program: Program, params: dict[str, torch.Tensor], world: int, rank: int):
    """(sharded Program, params) for ``rank`` of ``world``."""
    if world == 1:
        return program, params
    prog = copy.deepcopy(program)
    params = dict(params)
    tensors = prog.tensors
    producer = {o.tensor: k for k in prog.kernels for o in k.outputs}
    sharded: set[str] = set()

    attention_operands = {a.tensor for k in prog.kernels if k.kind == "attention" for a in k.args}

    def shard_cols(kspec, out_tensor: str):
        """Column-parallel: keep this rank's 1/world of the GEMM feeding out_tensor."""
        accs = _acc_of_output(kspec, next(o.value for o in kspec.outputs if o.tensor == out_tensor))
        # one accumulator behind two of q / k / v (a single wide GEMM split by columns): a contiguous
        # 1/world of its columns would hand this rank a mixed block of q, k and v heads
        for o in kspec.outputs:
            if o.tensor != out_tensor and o.tensor in attention_operands and _acc_of_output(kspec, o.value) & accs:
                raise TPError(f"{kspec.name}: {out_tensor} and {o.tensor} come from one accumulator; "
                              "compile q, k and v as separate GEMMs to shard them by heads")
        for g in kspec.gemms:
            if g.acc not in accs:
                continue
            arg = next(a for a in kspec.args if a.name == g.rhs)
            w = params[arg.tensor]
            n = w.shape[1]
            if n % world:
                raise TPError(f"{kspec.name}: width {n} is not divisible by {world}")
            c0, c1 = rank * n // world, (rank + 1) * n // world
            new = f"{arg.tensor}@tp{rank}/{world}"
            if new not in params:
                params[new] = w[:, c0:c1].contiguous()
                tensors[new] = TensorType((w.shape[0], c1 - c0), tensors[arg.tensor].dtype)
            arg.tensor = new

    def resize(name: str):
        t = tensors[name]
        if t.shape[1] % world:
            raise TPError(f"{name}: width {t.shape[1]} is not divisible by {world}")
        tensors[name] = TensorType((t.shape[0], t.shape[1] // world), t.dtype)

    # 1. attention: shard heads and the q/k/v producers
    for k in prog.kernels:
        if k.kind != "attention":
            continue
        a = k.attrs
        if a["heads"] % world or a.get("kv_heads", a["heads"]) % world:
            raise TPError(f"{k.name}: heads {a['heads']}/{a.get('kv_heads')} not divisible by {world}")
        for arg in k.args:
            if arg.cols:
                raise TPError(f"{k.name}: q/k/v must be whole tensors to shard")
            p = producer.get(arg.tensor)
            if p is None or p.kind != "gemm":
                raise TPError(f"{k.name}: {arg.role} is not produced by a GEMM kernel")
            if arg.tensor not in sharded:
                shard_cols(p, arg.tensor)
                resize(arg.tensor)
                sharded.add(arg.tensor)
        a["heads"] //= world
        a["kv_heads"] = a.get("kv_heads", a["heads"] * world) // world
        resize(k.outputs[0].tensor)
        sharded.add(k.outputs[0].tensor)
    # 2. SwiGLU GEMMs whose output feeds only GEMM LHSs: column-parallel
    lhs_of = {next(a.tensor for a in k.args if a.role == "lhs"): k for k in prog.kernels if k.kind == "gemm"}
    for k in prog.kernels:
        if k.kind != "gemm" or len(k.outputs) != 1 or len(k.gemms) != 2:
            continue
        ops = {o.name: o for o in k.epilogue}
        v = ops.get(k.outputs[0].value)
        is_swiglu = v is not None and v.op == "mul" and any(ops.get(i) is not None and ops[i].op == "silu" for i in v.inputs)
        if is_swiglu and k.outputs[0].tensor in lhs_of:
            shard_cols(k, k.outputs[0].tensor)
            resize(k.outputs[0].tensor)
            sharded.add(k.outputs[0].tensor)
    # row-scale broadcasts of column-parallel kernels keep their row count only
    for k in prog.kernels:
        if k.kind == "gemm" and any(o.tensor in sharded for o in k.outputs):
            for op in k.epilogue:
                if op.op == "broadcast":
                    op.attrs["shape"] = [op.attrs["shape"][0], -1]
    if not sharded:
        raise TPError("no attention heads or SwiGLU FFN to shard (tp_mode 'heads' applies to the Llama block)")
    # 3. row-parallel GEMMs: LHS sharded
    for k in prog.kernels:
        if k.kind != "gemm":
            continue
        lhs = next(a for a in k.args if a.role == "lhs")
        if lhs.tensor not in sharded:
            if any(a.tensor in sharded for a in k.args):
                raise TPError(f"{k.name}: reads a sharded tensor outside its LHS")
            continue
        if k.sumsq:
            raise TPError(f"{k.name}: RMSNorm over a sharded tensor needs its own reduction")
        for g in k.gemms:
            arg = next(a for a in k.args if a.name == g.rhs)
            w = params[arg.tensor]
            kk = w.shape[0]
            k0, k1 = rank * kk // world, (rank + 1) * kk // world
            new = f"{arg.tensor}@tp{rank}/{world}"
            if new not in params:
                params[new] = w[k0:k1, :].contiguous()
                tensors[new] = TensorType((k1 - k0, w.shape[1]), tensors[arg.tensor].dtype)
            arg.tensor = new
        k.k_extent //= world
        k.attrs["tp_allreduce"] = True
        if rank != 0:  # the residual is added once, by rank 0
            ops = {o.name: o for o in k.epilogue}
            extras = {a.name for a in k.args if a.role == "extra"}
            for o in k.outputs:
                node = ops.get(o.value)
                if node is not None and node.op == "add" and len(node.inputs) == 2:
                    keep = [i for i in node.inputs if i not in extras]
                    if len(keep) == 1:
                        o.value = keep[0]
                        k.epilogue = [e for e in k.epilogue if e.name != node.name]
                        k.args = [a for a in k.args if not (a.role == "extra" and a.name not in
                                                            {i for e in k.epilogue for i in e.inputs})]
    # every other kernel must read replicated tensors only
    for k in prog.kernels:
        if k.kind in ("gemm", "attention"):
            continue
        if any(a.tensor in sharded for a in k.args):
            raise TPError(f"{k.name} ({k.kind}) reads a sharded tensor")
    prog.params = sorted({a.tensor for k in prog.kernels for a in k.args if a.tensor in params})
    prog.metadata["tp"] = {"world": world, "rank": rank, "sharded": sorted(sharded)}
    return prog, params
