"""Launcher behaviour on the GPU that is not numerics of one kernel:

* a bounded device wait that is made to run out reports the timeout through
  the device error word instead of hanging (th_selftest_bounded_wait drives
  the same bounded mbarrier wait every pipelined kernel uses, with a
  microsecond limit and an arrival that comes late, not never);
* one process driving two GPUs: the launchers raise each kernel's
  shared-memory limit per device, so the large-shared-memory kernels launch on
  the second device too (skipped with one GPU).
"""

from __future__ import annotations

import math

import pytest
import torch

from conftest import rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    from torch_helion.b200 import lib

    lib.load()
    lib.device_error(clear=True)
    return lib


def test_bounded_wait_runs_out_and_reports(L):
    done = torch.full((1,), -1, dtype=torch.int32, device="cuda:0")
    # the barrier's only arrival comes 2 ms after the start; the wait gives up after 5 us
    L.selftest_bounded_wait(5_000, 2_000_000, done)
    torch.cuda.synchronize()
    assert int(done.item()) == 0
    assert L.device_error(clear=True) == 1  # TH_DEVERR_MBAR_TIMEOUT
    assert L.device_error(clear=True) == 0  # cleared by the previous read


def test_bounded_wait_sees_a_late_arrival_within_its_limit(L):
    done = torch.full((1,), -1, dtype=torch.int32, device="cuda:0")
    L.selftest_bounded_wait(50_000_000, 20_000, done)  # arrival after 20 us, limit 50 ms
    torch.cuda.synchronize()
    assert int(done.item()) == 1
    assert L.device_error(clear=True) == 0


def test_bounded_wait_rejects_out_of_range_limits(L):
    done = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    with pytest.raises(L.B200KernelError):
        L.selftest_bounded_wait(10, 0, done)
    with pytest.raises(L.B200KernelError):
        L.selftest_bounded_wait(1_000_000, 10**9, done)


def _gemm_once(L, dev):
    g = torch.Generator(device=dev).manual_seed(3)
    a = torch.randn(512, 768, device=dev, generator=g).bfloat16()
    w = torch.randn(1024, 768, device=dev, generator=g).bfloat16()
    out = torch.empty(512, 1024, device=dev, dtype=torch.bfloat16)
    L.gemm(a, w, out)
    ref = a.float() @ w.float().t()
    return rel_l2(out.float(), ref)


def _ssd_once(L, dev):
    g = torch.Generator(device=dev).manual_seed(4)
    b, s, h, p, n = 1, 512, 4, 64, 128
    x = torch.randn(b * s, h * p, device=dev, generator=g).bfloat16()
    B = torch.randn(b * s, n, device=dev, generator=g).bfloat16()
    C = torch.randn(b * s, n, device=dev, generator=g).bfloat16()
    dt = torch.rand(b * s, h, device=dev, generator=g) * 0.099 + 0.001
    A = -torch.exp(torch.rand(h, device=dev, generator=g) * math.log(16))
    out = torch.empty_like(x)
    L.ssd(x, dt, A, B, C, out, batch=b, seq=s, heads=h, head_dim=p, ngroups=1, state_dim=n, chunk=256)
    return out.float().cpu()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_launchers_alternate_between_two_devices(L):
    results = {}
    for dev in ("cuda:0", "cuda:1", "cuda:0", "cuda:1"):
        with torch.cuda.device(dev):
            assert _gemm_once(L, dev) < 1e-2
            results.setdefault(dev, []).append(_ssd_once(L, dev))
            torch.cuda.synchronize()
            assert L.device_error(clear=True) == 0
    # the same inputs give the same scan on either device, every time
    ref = results["cuda:0"][0]
    for outs in results.values():
        for o in outs:
            assert torch.equal(o, ref)
