"""th_ssd_noalloc: the allocation-free variant of the SSD scan.

Some callers cannot allocate device memory where they call the library: a
host framework that keeps every byte of device memory in its own pool and
does not let libraries call the CUDA allocator, a caller that cannot pay for
the synchronisation cudaFree implies, or a plugin handed only its input and
output pointers.  th_ssd_noalloc serves them with a fixed-size scratch array
inside the library instead of a caller-provided workspace.

This file is collected last (its name sorts after the other test files) so
that a run stopping at its first failure has already run everything else.
It is checked against the existing entry point th_ssd, through the C ABI,
on two calls in a row (the scratch keeps the previous call's contents).
"""

from __future__ import annotations

import ctypes
import math

import pytest
import torch

from conftest import rel_l2

pytestmark = pytest.mark.gpu


def _noalloc_fn():
    from torch_helion.b200 import lib

    l = lib.load()
    fn = l.th_ssd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(lib.SsdArgs), ctypes.c_void_p]
    return lib, fn


def _inputs(b, s, h, p, g, n, dtype, seed):
    torch.manual_seed(seed)
    t = b * s
    dev = torch.device("cuda:0")
    return dict(
        x=torch.randn(t, h * p, device=dev).to(dtype),
        B=torch.randn(t, g * n, device=dev).to(dtype),
        C=torch.randn(t, g * n, device=dev).to(dtype),
        z=torch.randn(t, h * p, device=dev).to(dtype),
        dt=torch.exp(torch.rand(t, h, device=dev) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3)),
        A=-torch.exp(torch.rand(h, device=dev) * math.log(16.0)),
        D=torch.ones(h, device=dev),
    )


def _args(lib, t, out, gss, b, s, h, p, g, n, chunk, dtype_code):
    a = lib.SsdArgs()
    a.x, a.ldx = t["x"].data_ptr(), t["x"].stride(0)
    a.dt, a.lddt = t["dt"].data_ptr(), t["dt"].stride(0)
    a.A = t["A"].data_ptr()
    a.B, a.ldb = t["B"].data_ptr(), t["B"].stride(0)
    a.C, a.ldc = t["C"].data_ptr(), t["C"].stride(0)
    a.D = t["D"].data_ptr()
    a.z, a.ldz = t["z"].data_ptr(), t["z"].stride(0)
    a.out, a.ldo = out.data_ptr(), out.stride(0)
    a.gss, a.ldgss = gss.data_ptr(), gss.stride(0)
    a.batch, a.seq, a.heads, a.head_dim, a.ngroups, a.state_dim, a.chunk = b, s, h, p, g, n, chunk
    a.dtype = dtype_code
    a.workspace, a.workspace_bytes = None, 0
    return a


@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 1e-2), (torch.float32, 1e-5)])
def test_noalloc_matches_th_ssd_on_two_calls(dtype, tol):
    lib, fn = _noalloc_fn()
    b, s, h, p, g, n, chunk = 2, 640, 8, 64, 1, 128, 256
    code = lib.TH_BF16 if dtype == torch.bfloat16 else lib.TH_F32
    for call in range(2):
        t = _inputs(b, s, h, p, g, n, dtype, seed=100 + call)
        ref = torch.empty_like(t["x"])
        ref_gss = torch.empty(b * s, h, device=ref.device)
        lib.ssd(t["x"], t["dt"], t["A"], t["B"], t["C"], ref, batch=b, seq=s, heads=h, head_dim=p, ngroups=g,
                state_dim=n, chunk=chunk, D=t["D"], z=t["z"], gss=ref_gss)
        out = torch.full_like(ref, float("nan"))
        gss = torch.full_like(ref_gss, float("nan"))
        a = _args(lib, t, out, gss, b, s, h, p, g, n, chunk, code)
        rc = fn(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
        assert rc == 0, lib.load().th_last_error_string().decode()
        torch.cuda.synchronize()
        assert rel_l2(out.float(), ref.float()) <= tol
        assert rel_l2(gss, ref_gss) <= 1e-5
    assert lib.device_error() == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib, fn = _noalloc_fn()
    b, s, h, p, g, n, chunk = 8, 4096, 64, 64, 1, 128, 256  # needs far more than the built-in scratch
    need = lib.ssd_workspace_size(b, s, h, p, n, chunk)
    t = {k: torch.empty(1, 1, device="cuda:0") for k in ("x", "B", "C", "z", "dt", "A", "D")}
    out = torch.empty(1, 1, device="cuda:0")
    gss = torch.empty(1, 64, device="cuda:0")
    a = _args(lib, t, out, gss, b, s, h, p, g, n, chunk, lib.TH_BF16)
    rc = fn(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    msg = lib.load().th_last_error_string().decode()
    assert need > (32 << 20)
    assert rc == -1 and "scratch" in msg and str(32 << 20) in msg
