"""ctypes binding of ``libth_b200.so`` (declared in ``include/th_b200.h``).

This module is the only place Python touches the C ABI.  Each wrapper takes
torch CUDA tensors, checks them, fills the argument struct with raw device
pointers and sizes, and launches on the current torch stream.  There is no
fallback: if the library is missing or a call fails, :class:`B200KernelError`
is raised with the library's own message.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

_PKG_ROOT = Path(__file__).resolve().parents[2]  # .../torch-helion_b200
LIB_PATH = Path(os.environ.get("TH_B200_LIB", _PKG_ROOT / "lib" / "libth_b200.so"))

TH_F32, TH_BF16, TH_F16 = 0, 1, 2
ACT_NONE, ACT_SILU, ACT_SOFTPLUS, ACT_GELU, ACT_GELU_TANH = 0, 1, 2, 3, 4
# activation name of a lowered GEMM plan -> TH_ACT_* code
ACT_CODES = {None: ACT_NONE, "identity": ACT_NONE, "silu": ACT_SILU, "softplus": ACT_SOFTPLUS, "gelu": ACT_GELU,
             "gelu_tanh": ACT_GELU_TANH}
_DTYPES = {torch.float32: TH_F32, torch.bfloat16: TH_BF16, torch.float16: TH_F16}

EXPORTED_SYMBOLS = (
    "th_last_error_string", "th_version", "th_device_error", "th_rowstat", "th_rmsnorm", "th_gemm",
    "th_attention", "th_conv1d", "th_ssd_workspace_size", "th_ssd", "th_embedding", "th_ssd_noalloc",
    "th_selftest_bounded_wait", "th_allreduce",
)


class B200KernelError(RuntimeError):
    """A C-ABI call returned an error status (or the library is missing)."""


_i64, _i32, _f32, _vp = ctypes.c_int64, ctypes.c_int32, ctypes.c_float, ctypes.c_void_p


class RowstatArgs(ctypes.Structure):
    _fields_ = [("x", _vp), ("ldx", _i64), ("sumsq", _vp), ("rows", _i64), ("cols", _i64), ("dtype", _i32)]


class RmsnormArgs(ctypes.Structure):
    _fields_ = [("x", _vp), ("ldx", _i64), ("gain", _vp), ("y", _vp), ("ldy", _i64), ("rows", _i64), ("cols", _i64),
                ("eps", _f32), ("dtype", _i32)]


class AllreduceArgs(ctypes.Structure):
    _fields_ = [("mc", _vp), ("peer_sig", _vp), ("sig", _vp), ("offset", _i64), ("bytes", _i64), ("dtype", _i32),
                ("rank", _i32), ("world", _i32), ("ctas", _i32), ("sumsq_mc", _vp), ("row_bytes", _i64)]


ALLREDUCE_SIGNAL_BYTES = 20480  # TH_ALLREDUCE_SIGNAL_BYTES
ALLREDUCE_MAX_CTAS = 256


class GemmArgs(ctypes.Structure):
    _fields_ = [
        ("a", _vp), ("lda", _i64), ("w", _vp), ("ldw", _i64), ("d", _vp), ("ldd", _i64),
        ("m", _i64), ("n", _i64), ("k", _i64), ("dtype", _i32),
        ("rs_parts", _vp), ("rs_nparts", _i32), ("rs_inv_k", _f32), ("rs_eps", _f32),
        ("act", _i32), ("act_begin", _i32), ("act_end", _i32), ("bias", _vp),
        ("rope_cos", _vp), ("rope_sin", _vp), ("rope_begin", _i32), ("rope_end", _i32), ("rope_head_dim", _i32),
        ("rope_seq", _i32),
        ("swiglu", _i32), ("residual", _vp), ("ld_res", _i64),
        ("out2", _vp), ("ld_out2", _i64), ("tail_begin", _i32),
        ("ss_out", _vp), ("ss_ld", _i64), ("sm_limit", _i32),
    ]


class AttentionArgs(ctypes.Structure):
    _fields_ = [("q", _vp), ("k", _vp), ("v", _vp), ("o", _vp), ("ldq", _i64), ("ldk", _i64), ("ldv", _i64),
                ("ldo", _i64), ("batch", _i32), ("seq", _i32), ("hq", _i32), ("hkv", _i32), ("head_dim", _i32),
                ("scale", _f32), ("causal", _i32), ("dtype", _i32)]


class Conv1dArgs(ctypes.Structure):
    _fields_ = [("x", _vp), ("ldx", _i64), ("w", _vp), ("bias", _vp), ("y", _vp), ("ldy", _i64), ("batch", _i32),
                ("seq", _i32), ("channels", _i32), ("width", _i32), ("act", _i32), ("dtype", _i32)]


class SsdArgs(ctypes.Structure):
    _fields_ = [
        ("x", _vp), ("ldx", _i64), ("dt", _vp), ("lddt", _i64), ("A", _vp), ("B", _vp), ("ldb", _i64),
        ("C", _vp), ("ldc", _i64), ("D", _vp), ("z", _vp), ("ldz", _i64), ("out", _vp), ("ldo", _i64),
        ("gss", _vp), ("ldgss", _i64),
        ("batch", _i32), ("seq", _i32), ("heads", _i32), ("head_dim", _i32), ("ngroups", _i32), ("state_dim", _i32),
        ("chunk", _i32), ("dtype", _i32), ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
    ]


class EmbeddingArgs(ctypes.Structure):
    _fields_ = [("ids", _vp), ("table", _vp), ("ldt", _i64), ("out", _vp), ("ldo", _i64), ("tokens", _i64),
                ("dim", _i64), ("vocab", _i64), ("dtype", _i32)]


_LIB: ctypes.CDLL | None = None


def _check_built_from_sources() -> None:
    """Refuse a library whose recorded source digest is not the digest of the
    sources beside it (torch-helion_b200/build.py writes it at build time)."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("_th_build", LIB_PATH.parents[1] / "build.py")
    if spec is None or spec.loader is None:
        return  # an installed copy without its build script: nothing to compare
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    if not (mod.CSRC.exists()):
        return
    have, want = mod.built_digest(), mod.source_digest()
    if have != want:
        raise B200KernelError(f"{LIB_PATH} was not built from the current sources (digest {have} != {want}): "
                              "rebuild with `python torch-helion_b200/build.py`")


def load() -> ctypes.CDLL:
    """Load the shared library once (raises if it has not been built)."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise B200KernelError(f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'`")
        _check_built_from_sources()
        lib = ctypes.CDLL(str(LIB_PATH))
        lib.th_last_error_string.restype = ctypes.c_char_p
        lib.th_version.restype = ctypes.c_char_p
        lib.th_ssd_workspace_size.restype = ctypes.c_size_t
        lib.th_ssd_workspace_size.argtypes = [_i32] * 6
        for name, st in (("th_rowstat", RowstatArgs), ("th_rmsnorm", RmsnormArgs), ("th_gemm", GemmArgs),
                         ("th_attention", AttentionArgs), ("th_conv1d", Conv1dArgs), ("th_ssd", SsdArgs),
                         ("th_ssd_noalloc", SsdArgs), ("th_embedding", EmbeddingArgs),
                         ("th_allreduce", AllreduceArgs)):
            fn = getattr(lib, name)
            fn.restype = ctypes.c_int
            fn.argtypes = [ctypes.POINTER(st), _vp]
        lib.th_device_error.restype = ctypes.c_int
        lib.th_device_error.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_int]
        lib.th_selftest_bounded_wait.restype = ctypes.c_int
        lib.th_selftest_bounded_wait.argtypes = [_i64, _i64, _vp, _vp]
        _LIB = lib
    return _LIB


def version() -> str:
    return load().th_version().decode()


def _check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().th_last_error_string().decode(errors="replace")
        raise B200KernelError(f"{what} failed with status {rc}: {msg}")


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _dt(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise B200KernelError(f"unsupported dtype {t.dtype}") from None


def _rows(t: torch.Tensor) -> tuple[int, int, int]:
    """(rows, cols, leading dimension) of a 2-D view with unit column stride."""
    if t.dim() != 2 or t.stride(1) != 1:
        raise B200KernelError(f"expected a 2-D row-major view, got shape {tuple(t.shape)} stride {t.stride()}")
    return t.shape[0], t.shape[1], t.stride(0)


def _cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise B200KernelError("all tensors must live on a CUDA device")


def device_error(clear: bool = True) -> int:
    """Device error word (non-zero: a kernel's bounded wait gave up)."""
    v = ctypes.c_int(0)
    _check(load().th_device_error(ctypes.byref(v), int(clear)), "th_device_error")
    return v.value


# ------------------------------------------------------------------ kernels
def allreduce(mc: int, peer_sig: torch.Tensor, sig: torch.Tensor, offset: int, nbytes: int, dtype: torch.dtype,
              rank: int, world: int, ctas: int = 0, sumsq_mc: int = 0, row_bytes: int = 0) -> None:
    """In-place multicast sum all-reduce of bytes [offset, offset + nbytes) of a symmetric buffer
    (th_allreduce): ``mc`` is the buffer's multicast address, ``peer_sig`` an int64 device tensor of
    every rank's signal-pad address, ``sig`` this rank's pad (uint8, zeroed before the first call).
    With ``sumsq_mc`` (multicast address of an fp32 per-row array) every reduced row's sum of
    squares is stored there too; each rank's slice must then be whole rows of ``row_bytes``."""
    if peer_sig.dtype != torch.int64 or peer_sig.numel() != world or not peer_sig.is_cuda:
        raise B200KernelError("allreduce: peer_sig must be an int64 CUDA tensor of world entries")
    if sig.numel() * sig.element_size() < ALLREDUCE_SIGNAL_BYTES:
        raise B200KernelError(f"allreduce: the signal pad needs {ALLREDUCE_SIGNAL_BYTES} bytes")
    a = AllreduceArgs(mc, peer_sig.data_ptr(), sig.data_ptr(), offset, nbytes, _DTYPES[dtype], rank, world, ctas,
                      sumsq_mc or None, row_bytes)
    _check(load().th_allreduce(ctypes.byref(a), _stream()), "th_allreduce")


def rowstat(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-row sum of squares (fp32)."""
    rows, cols, ld = _rows(x)
    out = torch.empty(rows, device=x.device, dtype=torch.float32) if out is None else out
    _cuda(x, out)
    a = RowstatArgs(x.data_ptr(), ld, out.data_ptr(), rows, cols, _dt(x))
    _check(load().th_rowstat(ctypes.byref(a), _stream()), "th_rowstat")
    return out


def rmsnorm(x: torch.Tensor, gain: torch.Tensor | None, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    rows, cols, ld = _rows(x)
    out = torch.empty_like(x) if out is None else out
    _, _, ldy = _rows(out)
    if gain is not None and (gain.dtype != torch.float32 or gain.numel() != cols):
        raise B200KernelError("rmsnorm gain must be fp32 [cols]")
    _cuda(x, out, gain)
    a = RmsnormArgs(x.data_ptr(), ld, _ptr(gain), out.data_ptr(), ldy, rows, cols, eps, _dt(x))
    _check(load().th_rmsnorm(ctypes.byref(a), _stream()), "th_rmsnorm")
    return out


def gemm(a: torch.Tensor, w: torch.Tensor, out: torch.Tensor, *, rs_parts: torch.Tensor | None = None,
         rs_inv_k: float = 1.0, rs_eps: float = 0.0, act: int = ACT_NONE, act_begin: int = 0, act_end: int = 0,
         bias: torch.Tensor | None = None, rope_cos: torch.Tensor | None = None, rope_sin: torch.Tensor | None = None,
         rope_begin: int = 0, rope_end: int = 0, rope_head_dim: int = 0, swiglu: bool = False,
         residual: torch.Tensor | None = None, out2: torch.Tensor | None = None, tail_begin: int = 0,
         ss_out: torch.Tensor | None = None, sm_limit: int = 0) -> torch.Tensor:
    """``out = epilogue(a @ w.T)``; see ``th_gemm`` in include/th_b200.h."""
    m, k, lda = _rows(a)
    n, k2, ldw = _rows(w)
    if k != k2:
        raise B200KernelError(f"gemm: K mismatch {k} vs {k2}")
    if w.dtype != a.dtype or out.dtype != a.dtype:
        raise B200KernelError("gemm: a, w and out must share a dtype")
    _, _, ldd = _rows(out)
    _cuda(a, w, out, rs_parts, bias, rope_cos, rope_sin, residual, out2, ss_out)
    args = GemmArgs()
    args.a, args.lda, args.w, args.ldw, args.d, args.ldd = a.data_ptr(), lda, w.data_ptr(), ldw, out.data_ptr(), ldd
    args.m, args.n, args.k, args.dtype = m, n, k, _dt(a)
    if rs_parts is not None:
        rp = rs_parts if rs_parts.dim() == 2 else rs_parts.reshape(-1, 1)
        if rp.dtype != torch.float32 or rp.shape[0] != m or not rp.is_contiguous():
            raise B200KernelError("gemm: rs_parts must be contiguous fp32 [m, nparts]")
        args.rs_parts, args.rs_nparts, args.rs_inv_k, args.rs_eps = rp.data_ptr(), rp.shape[1], rs_inv_k, rs_eps
    args.act, args.act_begin, args.act_end, args.bias = act, act_begin, act_end, _ptr(bias)
    if rope_cos is not None:
        args.rope_cos, args.rope_sin = rope_cos.data_ptr(), rope_sin.data_ptr()
        args.rope_begin, args.rope_end, args.rope_head_dim, args.rope_seq = rope_begin, rope_end, rope_head_dim, rope_cos.shape[0]
    args.swiglu = int(swiglu)
    if residual is not None:
        args.residual, args.ld_res = residual.data_ptr(), _rows(residual)[2]
    if out2 is not None:
        args.out2, args.ld_out2, args.tail_begin = out2.data_ptr(), _rows(out2)[2], tail_begin
    if ss_out is not None:
        args.ss_out, args.ss_ld = ss_out.data_ptr(), _rows(ss_out)[2]
    args.sm_limit = int(sm_limit)
    _check(load().th_gemm(ctypes.byref(args), _stream()), "th_gemm")
    return out


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, *, batch: int, seq: int, hq: int,
              hkv: int, head_dim: int, scale: float, causal: bool) -> torch.Tensor:
    _cuda(q, k, v, out)
    a = AttentionArgs(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), _rows(q)[2], _rows(k)[2], _rows(v)[2],
                      _rows(out)[2], batch, seq, hq, hkv, head_dim, scale, int(causal), _dt(q))
    _check(load().th_attention(ctypes.byref(a), _stream()), "th_attention")
    return out


def conv1d(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, *, batch: int, seq: int, act: int = ACT_SILU,
           bias: torch.Tensor | None = None) -> torch.Tensor:
    _, ch, ldx = _rows(x)
    if w.dtype != torch.float32 or w.dim() != 2 or w.shape[0] != ch or not w.is_contiguous():
        raise B200KernelError("conv1d: weight must be contiguous fp32 [channels, width]")
    _cuda(x, w, out, bias)
    a = Conv1dArgs(x.data_ptr(), ldx, w.data_ptr(), _ptr(bias), out.data_ptr(), _rows(out)[2], batch, seq, ch,
                   w.shape[1], act, _dt(x))
    _check(load().th_conv1d(ctypes.byref(a), _stream()), "th_conv1d")
    return out


def ssd_workspace_size(batch: int, seq: int, heads: int, head_dim: int, state_dim: int, chunk: int) -> int:
    return int(load().th_ssd_workspace_size(batch, seq, heads, head_dim, state_dim, chunk))


def _ssd_args(x, dt, A, B, C, out, batch, seq, heads, head_dim, ngroups, state_dim, chunk, D, z, gss) -> SsdArgs:
    if dt.dtype != torch.float32 or A.dtype != torch.float32 or (D is not None and D.dtype != torch.float32):
        raise B200KernelError("ssd: dt, A and D must be fp32")
    _cuda(x, dt, A, B, C, out, D, z, gss)
    a = SsdArgs()
    a.x, a.ldx = x.data_ptr(), _rows(x)[2]
    a.dt, a.lddt = dt.data_ptr(), _rows(dt)[2]
    a.A = A.data_ptr()
    a.B, a.ldb = B.data_ptr(), _rows(B)[2]
    a.C, a.ldc = C.data_ptr(), _rows(C)[2]
    a.D = _ptr(D)
    if z is not None:
        a.z, a.ldz = z.data_ptr(), _rows(z)[2]
    a.out, a.ldo = out.data_ptr(), _rows(out)[2]
    if gss is not None:
        a.gss, a.ldgss = gss.data_ptr(), _rows(gss)[2]
    a.batch, a.seq, a.heads, a.head_dim, a.ngroups, a.state_dim, a.chunk = batch, seq, heads, head_dim, ngroups, state_dim, chunk
    a.dtype = _dt(x)
    return a


def ssd(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, out: torch.Tensor, *,
        batch: int, seq: int, heads: int, head_dim: int, ngroups: int, state_dim: int, chunk: int = 256,
        D: torch.Tensor | None = None, z: torch.Tensor | None = None, gss: torch.Tensor | None = None,
        workspace: torch.Tensor | None = None) -> torch.Tensor:
    need = ssd_workspace_size(batch, seq, heads, head_dim, state_dim, chunk)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    _cuda(workspace)
    a = _ssd_args(x, dt, A, B, C, out, batch, seq, heads, head_dim, ngroups, state_dim, chunk, D, z, gss)
    a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    _check(load().th_ssd(ctypes.byref(a), _stream()), "th_ssd")
    return out


def ssd_noalloc(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, B: torch.Tensor, C: torch.Tensor,
                out: torch.Tensor, *, batch: int, seq: int, heads: int, head_dim: int, ngroups: int, state_dim: int,
                chunk: int = 256, D: torch.Tensor | None = None, z: torch.Tensor | None = None,
                gss: torch.Tensor | None = None) -> torch.Tensor:
    """th_ssd_noalloc: the same scan with the library's built-in scratch
    array instead of a caller workspace (no allocation on either side)."""
    a = _ssd_args(x, dt, A, B, C, out, batch, seq, heads, head_dim, ngroups, state_dim, chunk, D, z, gss)
    a.workspace, a.workspace_bytes = None, 0
    _check(load().th_ssd_noalloc(ctypes.byref(a), _stream()), "th_ssd_noalloc")
    return out


def selftest_bounded_wait(limit_ns: int, arrive_ns: int, completed: torch.Tensor) -> None:
    """Launch the bounded-wait self-test (see th_selftest_bounded_wait):
    ``completed`` (int32, one element, on the device) becomes 1 when the
    late arrival was seen within ``limit_ns``, else 0 with the device error
    word set."""
    if completed.dtype != torch.int32 or not completed.is_cuda:
        raise B200KernelError("selftest_bounded_wait: completed must be an int32 CUDA tensor")
    _check(load().th_selftest_bounded_wait(int(limit_ns), int(arrive_ns), completed.data_ptr(), _stream()),
           "th_selftest_bounded_wait")


def embedding(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    if ids.dtype != torch.int64:
        raise B200KernelError("embedding: ids must be int64")
    vocab, dim, ldt = _rows(table)
    _cuda(ids, table, out)
    a = EmbeddingArgs(ids.data_ptr(), table.data_ptr(), ldt, out.data_ptr(), _rows(out)[2], ids.numel(), dim, vocab,
                      _dt(table))
    _check(load().th_embedding(ctypes.byref(a), _stream()), "th_embedding")
    return out
