"""Lower OpIR KernelSpecs to B200 launch plans (and say which ones can't be).

This is the codegen seam of the reference (src/torch_helion/codegen/
emit.py:500-520 turns a KernelSpec into a Helion module; interpret.py:18-51
executes one): here a KernelSpec becomes a plan for one ``th_*`` C-ABI call
(``include/th_b200.h``).  A ``gemm`` spec's epilogue SSA is matched to the
fused stages of ``th_gemm``:

    out_segment = residual + act(rowscale * acc + bias)        (act: silu/softplus/gelu)
                | residual + rope(rowscale * acc)
                | residual + silu(rowscale * acc_gate) * (rowscale * acc_up)

Sibling GEMMs become column segments of one wide GEMM, ordered
[rope segments | plain | activation | fp32 tail].  Anything else raises
:class:`LoweringError`; the planner records that as an illegal candidate,
so no program ever reaches the GPU with an epilogue the kernels cannot run.
"""

from __future__ import annotations

from dataclasses import dataclass, field

from ..capture.opgraph import TensorType
from ..optimizer.opir import KernelArg, KernelSpec, Program


class LoweringError(RuntimeError):
    pass


@dataclass
class Segment:
    acc: str
    rhs: str            # program tensor of the [K, N] weight
    width: int
    output: str | None  # program tensor stored from this segment
    kind: str = "plain"  # plain | rope | act | tail


@dataclass
class GemmPlan:
    lhs: KernelArg
    segments: list[Segment]
    k: int
    rows: int
    rowscale: tuple[float, float] | None = None    # (inv_k, eps)
    act: str | None = None                         # "silu" | "softplus" | "gelu" | "gelu_tanh" | "identity" (bias only)
    bias: str | None = None                        # const tensor [w] of the act segment
    rope: tuple[str, str, int] | None = None       # (cos, sin, head_dim) const tensors [S, d]
    swiglu: tuple[str, str] | None = None          # (gate rhs, up rhs) for an interleaved weight
    swiglu_out: str | None = None
    residual: KernelArg | None = None
    outputs: dict[str, tuple[str, int, int]] = field(default_factory=dict)  # tensor -> (main|tail, c0, c1)
    n_main: int = 0
    n_tail: int = 0


@dataclass
class MacroPlan:
    kind: str
    args: dict[str, KernelArg]
    attrs: dict
    output: str


def _ep(spec: KernelSpec) -> dict:
    return {op.name: op for op in spec.epilogue}


def _parse_rowscale(spec: KernelSpec, ep: dict, col: str) -> tuple[float, float]:
    """powf(add(mul(sumsq, inv_k), eps), -0.5) -> (inv_k, eps)."""
    p = ep.get(col)
    if p is None or p.op != "powf" or p.attrs.get("scalar") != -0.5:
        raise LoweringError(f"{spec.name}: row scale {col} is not (.)^-0.5")
    a = ep.get(p.inputs[0])
    if a is None or a.op != "add" or "scalar" not in a.attrs:
        raise LoweringError(f"{spec.name}: row scale lacks the +eps term")
    m = ep.get(a.inputs[0])
    if m is None or m.op != "mul" or "scalar" not in m.attrs or m.inputs[0] != "sumsq":
        raise LoweringError(f"{spec.name}: row scale is not sumsq * 1/K")
    return float(m.attrs["scalar"]), float(a.attrs["scalar"])


def _scaled_acc(spec: KernelSpec, ep: dict, v: str, accs: set[str]):
    """(acc, rowscale) for ``acc`` or ``acc * broadcast(row scale)``."""
    if v in accs:
        return v, None
    node = ep.get(v)
    if node is not None and node.op == "mul" and len(node.inputs) == 2 and "scalar" not in node.attrs:
        for a, b in (node.inputs, node.inputs[::-1]):
            bn = ep.get(b)
            if a in accs and bn is not None and bn.op == "broadcast":
                return a, _parse_rowscale(spec, ep, bn.inputs[0])
    raise LoweringError(f"{spec.name}: {v} is not a (row-scaled) accumulator")


def lower_gemm(spec: KernelSpec, tensors: dict[str, TensorType], fp32_outputs: set[str]) -> GemmPlan:
    ep = _ep(spec)
    args = {a.name: a for a in spec.args}
    accs = {g.acc: g for g in spec.gemms}
    rhs_of = {g.acc: args[g.rhs].tensor for g in spec.gemms}
    width = {acc: tensors[rhs_of[acc]].shape[1] for acc in accs}
    plan = GemmPlan(lhs=args["lhs"], segments=[], k=spec.k_extent, rows=spec.grid["rows"])
    seg_of: dict[str, Segment] = {}
    scales = set()
    for out in spec.outputs:
        v = out.value
        node = ep.get(v)
        # residual (outermost add of a DRAM tensor of the output's shape)
        if node is not None and node.op == "add" and len(node.inputs) == 2 and "scalar" not in node.attrs:
            for a, b in (node.inputs, node.inputs[::-1]):
                if b in args and args[b].role == "extra" and b not in accs:
                    if plan.residual is not None:
                        raise LoweringError(f"{spec.name}: more than one residual")
                    plan.residual = args[b]
                    v, node = a, ep.get(a)
                    break
        # swiglu
        if node is not None and node.op == "mul" and len(node.inputs) == 2 and "scalar" not in node.attrs:
            for a, b in (node.inputs, node.inputs[::-1]):
                an = ep.get(a)
                if an is not None and an.op == "silu":
                    try:
                        ga, gs = _scaled_acc(spec, ep, an.inputs[0], set(accs))
                        ua, us = _scaled_acc(spec, ep, b, set(accs))
                    except LoweringError:
                        continue
                    if len(accs) != 2 or len(spec.outputs) != 1 or width[ga] != width[ua] or width[ga] % 64:
                        raise LoweringError(f"{spec.name}: SwiGLU needs exactly a gate and an up GEMM of equal width (multiple of 64)")
                    scales.update({gs, us})
                    plan.swiglu = (rhs_of[ga], rhs_of[ua])
                    plan.swiglu_out = out.tensor
                    plan.segments = [Segment(ga, rhs_of[ga], width[ga], None, "swiglu"),
                                     Segment(ua, rhs_of[ua], width[ua], None, "swiglu")]
                    v = None
                    break
            if v is None:
                continue
        kind, act, bias, rope = "plain", None, None, None
        if node is not None and node.op in ("silu", "softplus", "gelu"):
            act = node.op if node.op != "gelu" or node.attrs.get("approximate", "none") == "none" else "gelu_tanh"
            v, node = node.inputs[0], ep.get(node.inputs[0])
            if node is not None and node.op == "add" and len(node.inputs) == 2 and "scalar" not in node.attrs:
                for a, b in (node.inputs, node.inputs[::-1]):
                    if b in args and args[b].role == "const" and tensors[args[b].tensor].numel == width.get(
                            _acc_below(spec, ep, a, set(accs)), -1):
                        bias = args[b].tensor
                        v, node = a, ep.get(a)
                        break
            kind = "act"
        elif node is not None and node.op == "add" and len(node.inputs) == 2 and "scalar" not in node.attrs:
            # a bias without an activation (a Linear's bias): an identity activation segment
            for a, b in (node.inputs, node.inputs[::-1]):
                if b in args and args[b].role == "const" and tensors[args[b].tensor].numel == width.get(
                        _acc_below(spec, ep, a, set(accs)), -1):
                    act, bias, kind = "identity", args[b].tensor, "act"
                    v, node = a, ep.get(a)
                    break
        elif node is not None and node.op == "rope":
            x, c, s = node.inputs
            if args.get(c) is None or args.get(s) is None:
                raise LoweringError(f"{spec.name}: rope tables must be constants")
            rope = (args[c].tensor, args[s].tensor, int(node.attrs["head_dim"]))
            v, node = x, ep.get(x)
            kind = "rope"
        acc, scale = _scaled_acc(spec, ep, v, set(accs))
        scales.add(scale)
        if acc in seg_of:
            raise LoweringError(f"{spec.name}: accumulator {acc} stored twice")
        if kind == "act":
            if plan.act is not None:
                raise LoweringError(f"{spec.name}: more than one activation segment")
            plan.act, plan.bias = act, bias
            if out.tensor in fp32_outputs:
                kind = "tail"
        if kind == "rope":
            if plan.rope is not None and plan.rope != rope:
                raise LoweringError(f"{spec.name}: rope segments with different tables")
            plan.rope = rope
        seg = Segment(acc, rhs_of[acc], width[acc], out.tensor, kind)
        seg_of[acc] = seg
    if plan.swiglu is None:
        if set(seg_of) != set(accs):
            missing = set(accs) - set(seg_of)
            raise LoweringError(f"{spec.name}: accumulators {sorted(missing)} are not stored")
        rank = {"rope": 0, "plain": 1, "act": 2, "tail": 3}
        plan.segments = sorted(seg_of.values(), key=lambda s: rank[s.kind])
    if len(scales) != 1:
        raise LoweringError(f"{spec.name}: segments disagree on the row scale")
    plan.rowscale = scales.pop()
    if plan.rowscale is not None and not spec.sumsq:
        raise LoweringError(f"{spec.name}: row scale without the sumsq fold")
    # column layout
    c = 0
    for seg in plan.segments:
        if seg.kind == "tail":
            continue
        if seg.output is not None:
            plan.outputs[seg.output] = ("main", c, c + seg.width)
        c += seg.width
    plan.n_main = c if plan.swiglu is None else plan.segments[0].width
    if plan.swiglu is not None:
        plan.outputs[plan.swiglu_out] = ("main", 0, plan.n_main)
    t = 0
    for seg in plan.segments:
        if seg.kind == "tail":
            plan.outputs[seg.output] = ("tail", t, t + seg.width)
            t += seg.width
    plan.n_tail = t
    # what th_gemm needs
    if plan.n_main % 8 or (plan.n_tail and plan.n_main % 8):
        raise LoweringError(f"{spec.name}: output width {plan.n_main} is not a multiple of 8")
    if plan.rope is not None:
        hd = plan.rope[2]
        if hd % 2 or hd > 128 or 128 % hd:
            raise LoweringError(f"{spec.name}: rope head_dim {hd} must divide 128")
        rc = 0
        for seg in plan.segments:
            if seg.kind == "rope" and (rc % hd or seg.width % hd):
                raise LoweringError(f"{spec.name}: rope segment not aligned to head_dim")
            rc += seg.width if seg.kind != "tail" else 0
    if plan.residual is not None:
        if len(spec.outputs) != 1:
            raise LoweringError(f"{spec.name}: a residual must cover the whole output")
    if spec.k_extent % 8:
        raise LoweringError(f"{spec.name}: K={spec.k_extent} must be a multiple of 8 (16-byte TMA rows)")
    return plan


def _acc_below(spec: KernelSpec, ep: dict, v: str, accs: set[str]) -> str | None:
    try:
        return _scaled_acc(spec, ep, v, accs)[0]
    except LoweringError:
        return None


def lower_macro(spec: KernelSpec, tensors: dict[str, TensorType]) -> MacroPlan:
    args = {a.role: a for a in spec.args}
    a = spec.attrs
    if spec.kind == "attention":
        if a["head_dim"] not in (16, 32, 64, 128):
            raise LoweringError(f"{spec.name}: head_dim {a['head_dim']} not built")
        if a["heads"] % a.get("kv_heads", a["heads"]):
            raise LoweringError(f"{spec.name}: heads not a multiple of kv_heads")
    elif spec.kind == "ssd":
        if a["head_dim"] > 64 or a["head_dim"] % 4 or a["state_dim"] > 256 or a["head_dim"] * a["state_dim"] > 16384:
            raise LoweringError(f"{spec.name}: ssd head_dim {a['head_dim']} / state {a['state_dim']} not built")
        if a["heads"] % a["ngroups"]:
            raise LoweringError(f"{spec.name}: heads not a multiple of ngroups")
    elif spec.kind == "causal_conv1d":
        ch = tensors[spec.outputs[0].tensor].shape[1]
        if ch % 8 or a["width"] not in (2, 3, 4):
            raise LoweringError(f"{spec.name}: conv channels {ch} / width {a['width']} not built")
    elif spec.kind in ("rmsnorm", "embedding"):
        pass
    else:
        raise LoweringError(f"{spec.name}: unknown kernel kind {spec.kind}")
    return MacroPlan(spec.kind, args, dict(a), spec.outputs[0].tensor)


def fp32_outputs(program: Program) -> set[str]:
    """Tensors a consumer needs in fp32 (the scan's dt)."""
    return {a.tensor for k in program.kernels if k.kind == "ssd" for a in k.args if a.role == "dt"}


def lower_kernel(spec: KernelSpec, program: Program):
    if spec.kind == "gemm":
        return lower_gemm(spec, program.tensors, fp32_outputs(program))
    return lower_macro(spec, program.tensors)


def check_lowering(program: Program) -> list[str]:
    """Violations (empty = every kernel has a B200 launch)."""
    out = []
    f32 = fp32_outputs(program)
    for spec in program.kernels:
        try:
            if spec.kind == "gemm":
                lower_gemm(spec, program.tensors, f32)
            else:
                lower_macro(spec, program.tensors)
        except LoweringError as e:
            out.append(str(e))
    for k in program.kernels:
        if k.kind == "ssd":
            dt = next(a for a in k.args if a.role == "dt")
            prod = program.producer(dt.tensor)
            if prod is None or prod.kind != "gemm":
                out.append(f"{k.name}: dt must come from a GEMM epilogue (fp32 tail)")
    return out
