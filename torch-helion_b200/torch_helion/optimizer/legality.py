"""Kernel legality for the B200 backend.

The reference checks Loom's structural constraints C2-C5 per kernel (one
reduction loop, 32-aligned extents, registered epilogue ops, operand shapes
that match the output tile; src/torch_helion/optimizer/legality.py:56-138).
Here the constraints are those of the ``th_*`` launches the kernels lower to
(``include/th_b200.h``), checked in two layers:

* structural rules, named so a rejected planner candidate says which one it
  broke:

  ``operands``   every argument and output names a declared tensor, and a
                 column view lies inside its tensor;
  ``gemm-shape`` the left operand is [rows, K], every weight [K, n], the grid
                 covers rows x sum(n), every output has the grid's rows;
  ``dtype``      GEMM operands share one dtype, and it is fp32, bf16 or fp16;
                 attention q, k and v share one dtype;
  ``attention``  q is [batch*seq, heads*head_dim], k and v
                 [batch*seq, kv_heads*head_dim], heads a multiple of kv_heads;
  ``ssd``        x is [batch*seq, heads*head_dim], B and C
                 [batch*seq, ngroups*state_dim], dt has one column per head,
                 heads a multiple of ngroups;
  ``conv``       the taps have one row per channel and the output the input's
                 width;

* ``lowering``: the kernel maps onto one C-ABI call
  (:func:`torch_helion.b200.lower.check_lowering`: the GEMM epilogue matches
  th_gemm's fused stages, head dims, state sizes and conv widths that were
  built, the scan's dt produced by a GEMM epilogue in fp32).

A legal program may still run a kernel on a slower device path (fp32 GEMMs on
the SIMT kernel, attention head dims other than 64/128 on the SIMT flash
kernel, SSD shapes other than head_dim 64 / chunk 256 / d_state 64-256 on the
three-pass scan, column views that do not start on a 16-byte boundary).  The
report lists those as ``notes``; they never make a program illegal.
"""

from __future__ import annotations

from dataclasses import dataclass, field

from .opir import KernelArg, KernelSpec, Program

_DTYPES = ("float32", "bfloat16", "float16")
_TWO_BYTE = ("bfloat16", "float16")


@dataclass
class Violation:
    kernel: str
    rule: str
    message: str

    def __str__(self) -> str:
        return f"[{self.kernel}] {self.rule}: {self.message}"


@dataclass
class LegalityReport:
    violations: list[Violation] = field(default_factory=list)
    notes: list[str] = field(default_factory=list)  # legal but slower device paths

    @property
    def ok(self) -> bool:
        return not self.violations

    def add(self, kernel: str, rule: str, message: str) -> None:
        self.violations.append(Violation(kernel, rule, message))

    def note(self, kernel: str, message: str) -> None:
        self.notes.append(f"[{kernel}] {message}")

    def __str__(self) -> str:
        return "legal" if self.ok else "\n".join(str(v) for v in self.violations)


def _width(arg: KernelArg, shape: tuple[int, ...]) -> int:
    """Columns an argument covers: its column view, else its tensor's last dimension."""
    if arg.cols is not None:
        return arg.cols[1] - arg.cols[0]
    return shape[-1] if shape else 1


def _check_operands(spec: KernelSpec, program: Program, rep: LegalityReport) -> bool:
    ok = True
    for a in spec.args:
        t = program.tensors.get(a.tensor)
        if t is None:
            rep.add(spec.name, "operands", f"argument {a.name} names undeclared tensor {a.tensor}")
            ok = False
        elif a.cols is not None:
            c0, c1 = a.cols
            if not (0 <= c0 < c1 <= (t.shape[-1] if t.shape else 1)):
                rep.add(spec.name, "operands", f"column view {a.cols} of {a.tensor} lies outside its {t.shape}")
                ok = False
    for o in spec.outputs:
        if o.tensor not in program.tensors:
            rep.add(spec.name, "operands", f"output {o.value} names undeclared tensor {o.tensor}")
            ok = False
    return ok


def _check_gemm(spec: KernelSpec, program: Program, rep: LegalityReport) -> None:
    k, T = spec.name, program.tensors
    lhs = next((a for a in spec.args if a.role == "lhs"), None)
    rhs = [a for a in spec.args if a.role == "rhs"]
    if lhs is None or not rhs:
        rep.add(k, "gemm-shape", "a GEMM kernel needs a left operand and at least one weight")
        return
    K, rows = spec.k_extent, spec.grid.get("rows")
    lt = T[lhs.tensor]
    if len(lt.shape) != 2 or _width(lhs, lt.shape) != K:
        rep.add(k, "gemm-shape", f"left operand {lhs.tensor} {lt.shape} does not have K = {K} columns")
    if len(lt.shape) == 2 and rows != lt.shape[0]:
        rep.add(k, "gemm-shape", f"grid rows {rows} differ from the left operand's {lt.shape[0]}")
    n_total = 0
    for a in rhs:
        s = T[a.tensor].shape
        if len(s) != 2 or s[0] != K:
            rep.add(k, "gemm-shape", f"weight {a.tensor} {s} is not [K = {K}, n]")
        else:
            n_total += s[1]
    if spec.grid.get("cols") not in (None, n_total):
        rep.add(k, "gemm-shape", f"grid columns {spec.grid.get('cols')} differ from the weights' {n_total}")
    for o in spec.outputs:
        s = T[o.tensor].shape
        if len(s) != 2 or s[0] != rows:
            rep.add(k, "gemm-shape", f"output {o.tensor} {s} does not have the grid's {rows} rows")
    dts = {T[a.tensor].dtype for a in [lhs, *rhs]}
    if len(dts) > 1:
        rep.add(k, "dtype", f"left operand and weights mix dtypes {sorted(dts)}")
    elif dts and next(iter(dts)) not in _DTYPES:
        rep.add(k, "dtype", f"GEMM dtype {next(iter(dts))} has no kernel (fp32, bf16 or fp16)")
    dt = next(iter(dts)) if len(dts) == 1 else None
    if dt == "float32":
        rep.note(k, "fp32 GEMM: SIMT kernel (tf32 tensor cores cannot meet the fp32 bound)")
    elif dt in _TWO_BYTE and rows is not None and rows <= 128:
        rep.note(k, "at most 128 rows: single-CTA tcgen05 kernel instead of CTA pairs")
    if lhs.cols is not None and lhs.cols[0] * 2 % 16:
        rep.note(k, f"left operand view starts at column {lhs.cols[0]}, not on a 16-byte boundary")


def _check_attention(spec: KernelSpec, program: Program, rep: LegalityReport) -> None:
    k, T, a = spec.name, program.tensors, spec.attrs
    heads, kvh, d = a["heads"], a.get("kv_heads", a["heads"]), a["head_dim"]
    rows = a["batch"] * a["seq"]
    if heads % kvh:
        rep.add(k, "attention", f"{heads} query heads are not a multiple of {kvh} key/value heads")
    want = {"q": heads * d, "k": kvh * d, "v": kvh * d}
    dts = set()
    for arg in spec.args:
        if arg.role not in want:
            continue
        s = T[arg.tensor].shape
        dts.add(T[arg.tensor].dtype)
        if len(s) != 2 or s[0] != rows or _width(arg, s) != want[arg.role]:
            n = heads if arg.role == "q" else kvh
            rep.add(k, "attention", f"{arg.role} operand {arg.tensor} {s} is not [batch*seq = {rows}, "
                                    f"{n} heads x head_dim {d} = {want[arg.role]}]")
        elif arg.cols is not None and arg.cols[0] * 2 % 16:
            rep.note(k, f"{arg.role} view starts at column {arg.cols[0]}: not a TMA operand, SIMT flash kernel")
    if len(dts) > 1:
        rep.add(k, "dtype", f"q, k and v mix dtypes {sorted(dts)}")
    dt = next(iter(dts)) if len(dts) == 1 else None
    if dt not in _TWO_BYTE or d not in (64, 128):
        rep.note(k, f"{dt} head_dim {d}: SIMT flash kernel (tcgen05 path: bf16/fp16, head_dim 64 or 128)")


def _check_ssd(spec: KernelSpec, program: Program, rep: LegalityReport) -> None:
    k, T, a = spec.name, program.tensors, spec.attrs
    rows = a["batch"] * a["seq"]
    want = {"x": a["heads"] * a["head_dim"], "B": a["ngroups"] * a["state_dim"],
            "C": a["ngroups"] * a["state_dim"], "dt": a["heads"]}
    if a["heads"] % a["ngroups"]:
        rep.add(k, "ssd", f"{a['heads']} heads are not a multiple of {a['ngroups']} B/C groups")
    dt = None
    for arg in spec.args:
        if arg.role not in want:
            continue
        s = T[arg.tensor].shape
        if arg.role == "x":
            dt = T[arg.tensor].dtype
        if len(s) != 2 or s[0] != rows or _width(arg, s) != want[arg.role]:
            rep.add(k, "ssd", f"{arg.role} operand {arg.tensor} {s} is not [{rows}, {want[arg.role]}]")
    if not (dt in _TWO_BYTE and a["head_dim"] == 64 and a["chunk"] == 256 and a["state_dim"] in (64, 128, 256)):
        rep.note(k, f"{dt} head_dim {a['head_dim']} chunk {a['chunk']} d_state {a['state_dim']}: three-pass scan "
                    "(tcgen05 chunk path: bf16/fp16, head_dim 64, chunk 256, d_state 64/128/256)")


def _check_conv(spec: KernelSpec, program: Program, rep: LegalityReport) -> None:
    k, T = spec.name, program.tensors
    x = next((a for a in spec.args if a.role == "x"), None)
    w = next((a for a in spec.args if a.role == "w"), None)
    if x is None or w is None or not spec.outputs:
        rep.add(k, "conv", "a causal conv needs an input, taps and an output")
        return
    ch = _width(x, T[x.tensor].shape)
    if T[w.tensor].shape[0] != ch:
        rep.add(k, "conv", f"taps {w.tensor} {T[w.tensor].shape} do not have one row per channel ({ch})")
    out = T[spec.outputs[0].tensor].shape
    if out[-1] != ch:
        rep.add(k, "conv", f"output {spec.outputs[0].tensor} {out} does not have the input's {ch} channels")
    if T[x.tensor].dtype not in _TWO_BYTE:
        rep.note(k, "fp32 causal conv: SIMT kernel (TMA-staged kernel: bf16/fp16)")


_KIND_RULES = {"gemm": _check_gemm, "attention": _check_attention, "ssd": _check_ssd,
               "causal_conv1d": _check_conv}


def check_kernel(spec: KernelSpec, program: Program, report: LegalityReport | None = None) -> LegalityReport:
    """The structural rules for one kernel (the lowering check needs the whole program)."""
    rep = report if report is not None else LegalityReport()
    if _check_operands(spec, program, rep):
        rule = _KIND_RULES.get(spec.kind)
        if rule is not None:
            rule(spec, program, rep)
    return rep


def check_program(program: Program) -> LegalityReport:
    """Every kernel's structural rules, then the lowering check; the planner
    records the violations of an illegal candidate and skips it."""
    from ..b200.lower import check_lowering

    rep = LegalityReport()
    for spec in program.kernels:
        check_kernel(spec, program, rep)
    if rep.ok:  # lowering assumes well-formed operands
        for msg in check_lowering(program):
            kname = msg.split(":", 1)[0]
            rep.add(kname, "lowering", msg.split(":", 1)[1].strip() if ":" in msg else msg)
    return rep
