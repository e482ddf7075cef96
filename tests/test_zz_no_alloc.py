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

import math

import pytest
import torch

from conftest import rel_l2

pytestmark = pytest.mark.gpu


def _lib():
    from torch_helion.b200 import lib

    lib.load()
    return lib


def _inputs(b, s, h, p, g, n, dtype, seed, device="cuda:0"):
    torch.manual_seed(seed)
    t = b * s
    dev = torch.device(device)
    return dict(
        x=torch.randn(t, h * p, device=dev).to(dtype),
        B=torch.randn(t, g * n, device=dev).to(dtype),
        C=torch.randn(t, g * n, device=dev).to(dtype),
        z=torch.randn(t, h * p, device=dev).to(dtype),
        dt=torch.exp(torch.rand(t, h, device=dev) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3)),
        A=-torch.exp(torch.rand(h, device=dev) * math.log(16.0)),
        D=torch.ones(h, device=dev),
    )


def _both(lib, t, b, s, h, p, g, n, chunk):
    """(th_ssd output, gss) and (th_ssd_noalloc output, gss) on the same inputs;
    the no-alloc outputs start as NaN so nothing stale can pass."""
    kw = dict(batch=b, seq=s, heads=h, head_dim=p, ngroups=g, state_dim=n, chunk=chunk, D=t["D"], z=t["z"])
    ref = torch.empty_like(t["x"])
    ref_gss = torch.empty(b * s, h, device=ref.device)
    lib.ssd(t["x"], t["dt"], t["A"], t["B"], t["C"], ref, gss=ref_gss, **kw)
    out = torch.full_like(ref, float("nan"))
    gss = torch.full_like(ref_gss, float("nan"))
    lib.ssd_noalloc(t["x"], t["dt"], t["A"], t["B"], t["C"], out, gss=gss, **kw)
    torch.cuda.synchronize(ref.device)
    return (ref, ref_gss), (out, gss)


# (b, s, h, p, g, n, chunk): the chunk-256 tcgen05 path at every state size
# (128: serial chunk walk; 64 and 256: chunk-parallel states + state pass),
# the mma.sync path (head_dim 32, chunk 128) and, in fp32, the SIMT path
SHAPES = {
    "tc_state128": (2, 640, 8, 64, 1, 128, 256),
    "tc_state64": (2, 640, 8, 64, 1, 64, 256),
    "tc_state256": (1, 700, 4, 64, 1, 256, 256),
    "mma_hd32_chunk128": (2, 384, 6, 32, 2, 64, 128),
}


@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 1e-2), (torch.float16, 1e-2), (torch.float32, 1e-5)],
                         ids=["bf16", "fp16", "fp32"])
@pytest.mark.parametrize("shape", list(SHAPES), ids=list(SHAPES))
def test_noalloc_matches_th_ssd_on_two_calls(shape, dtype, tol):
    lib = _lib()
    b, s, h, p, g, n, chunk = SHAPES[shape]
    for call in range(2):  # the scratch keeps the first call's contents when the second runs
        t = _inputs(b, s, h, p, g, n, dtype, seed=100 + call)
        (ref, ref_gss), (out, gss) = _both(lib, t, b, s, h, p, g, n, chunk)
        assert rel_l2(out.float(), ref.float()) <= tol
        assert rel_l2(gss, ref_gss) <= 1e-5
    assert lib.device_error() == 0


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_noalloc_on_a_second_device():
    """Each GPU that loads the library has its own copy of the scratch array;
    a call on cuda:1 after cuda:0 (one process) uses cuda:1's copy."""
    lib = _lib()
    b, s, h, p, g, n, chunk = SHAPES["tc_state128"]
    for dev in ("cuda:0", "cuda:1", "cuda:0"):
        with torch.cuda.device(dev):
            t = _inputs(b, s, h, p, g, n, torch.bfloat16, seed=7, device=dev)
            (ref, ref_gss), (out, gss) = _both(lib, t, b, s, h, p, g, n, chunk)
            assert rel_l2(out.float(), ref.float()) <= 1e-2
            assert lib.device_error() == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from torch_helion.b200 import lib

    b, s, h, p, g, n, chunk = 8, 4096, 64, 64, 1, 128, 256  # needs far more than the built-in scratch
    need = lib.ssd_workspace_size(b, s, h, p, n, chunk)
    assert need > (32 << 20)
    t = {k: torch.empty(1, 1, device="cuda:0") for k in ("x", "B", "C", "z")}
    with pytest.raises(lib.B200KernelError) as e:
        lib.ssd_noalloc(t["x"].bfloat16(), torch.empty(1, 1, device="cuda:0"), torch.empty(64, device="cuda:0"),
                        t["B"].bfloat16(), t["C"].bfloat16(), torch.empty(1, 1, device="cuda:0").bfloat16(),
                        batch=b, seq=s, heads=h, head_dim=p, ngroups=g, state_dim=n, chunk=chunk)
    msg = str(e.value)
    assert "status -1" in msg and "scratch" in msg and str(32 << 20) in msg
