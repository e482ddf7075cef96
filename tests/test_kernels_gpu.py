"""Per-kernel numerics on the GPU: every C-ABI entry point against a plain
PyTorch fp32 statement of the same op (the kernels are floating point, so a
torch fp32 reference is the checker here; model-level parity against the
oracle lives in test_parity_gpu.py).

Tolerances (rel-L2 unless stated): fp32 kernels <= 1e-5; bf16/fp16 outputs
<= 1e-2 (one rounding of the output to 8/11 mantissa bits dominates).
"""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 1e-2, torch.float16: 5e-3}


@pytest.fixture(scope="module")
def L():
    from torch_helion.b200 import lib

    lib.load()
    return lib


def _dev():
    return torch.device("cuda:0")


# ----------------------------------------------------------------- rows
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rows,cols", [(1, 8), (37, 768), (1000, 4096), (5, 13)])
def test_rowstat(L, dtype, rows, cols):
    torch.manual_seed(0)
    x = torch.randn(rows, cols, device=_dev()).to(dtype)
    s = L.rowstat(x)
    ref = (x.float() ** 2).sum(-1)
    assert rel_l2(s, ref) < 1e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_rmsnorm(L, dtype):
    torch.manual_seed(0)
    x = torch.randn(333, 1024, device=_dev()).to(dtype)
    g = torch.rand(1024, device=_dev()) + 0.5
    y = L.rmsnorm(x, g, 1e-5)
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5) * g
    assert rel_l2(y.float(), ref) < TOL[dtype]


# ----------------------------------------------------------------- gemm
def _gemm_ref(a, w):
    return a.float() @ w.float().t()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("m,n,k", [(128, 128, 64), (300, 384, 200), (512, 1024, 1024), (64, 136, 72), (1000, 3352, 768)])
def test_gemm_plain(L, dtype, m, n, k):
    torch.manual_seed(1)
    a = torch.randn(m, k, device=_dev()).to(dtype)
    w = (torch.randn(n, k, device=_dev()) * 0.05).to(dtype)
    out = torch.empty(m, n, device=_dev(), dtype=dtype)
    L.gemm(a, w, out)
    torch.cuda.synchronize()
    assert L.device_error() == 0
    assert rel_l2(out.float(), _gemm_ref(a, w)) < TOL[dtype]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gemm_rowscale_residual_sumsq(L, dtype):
    """RMSNorm row scale from rowstat partials, residual add, and the
    sum-of-squares partials of the stored output."""
    torch.manual_seed(2)
    m, n, k = 257, 512, 256
    x = torch.randn(m, k, device=_dev()).to(dtype)
    w = (torch.randn(n, k, device=_dev()) * 0.05).to(dtype)
    res = torch.randn(m, n, device=_dev()).to(dtype)
    parts = L.rowstat(x).reshape(m, 1)
    out = torch.empty(m, n, device=_dev(), dtype=dtype)
    ss = torch.zeros(m, n // 64, device=_dev())
    L.gemm(x, w, out, rs_parts=parts, rs_inv_k=1.0 / k, rs_eps=1e-6, residual=res, ss_out=ss)
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)
    ref = (xf @ w.float().t()) * r + res.float()
    assert rel_l2(out.float(), ref) < TOL[dtype]
    ss_ref = out.float().pow(2).reshape(m, n // 64, 64).sum(-1)
    assert rel_l2(ss, ss_ref) < 1e-5


@pytest.mark.parametrize("m,n,k", [(4000, 800, 512), (300, 1000, 256), (8192, 4096, 512), (96, 768, 128)])
def test_gemm_residual_widths(L, m, n, k):
    """Residual epilogue across output widths: whole 32-column chunks (the residual arrives by TMA
    into the staging buffer), a last column tile that is mostly past the output (n = 800), a width
    that is not a multiple of 32 (per-lane residual loads), ragged rows and a single row tile."""
    torch.manual_seed(9)
    dt = torch.bfloat16
    x = torch.randn(m, k, device=_dev()).to(dt)
    w = (torch.randn(n, k, device=_dev()) * 0.05).to(dt)
    res = torch.randn(m, n, device=_dev()).to(dt)
    out = torch.empty(m, n, device=_dev(), dtype=dt)
    ss = torch.zeros(m, (n + 63) // 64, device=_dev())
    L.gemm(x, w, out, residual=res, ss_out=ss)
    torch.cuda.synchronize()
    assert L.device_error() == 0
    assert rel_l2(out.float(), _gemm_ref(x, w) + res.float()) < TOL[dt]
    o = out.float()
    pad = (64 - n % 64) % 64
    ss_ref = F.pad(o, (0, pad)).pow(2).reshape(m, -1, 64).sum(-1)
    assert rel_l2(ss, ss_ref) < 1e-5


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gemm_softplus_tail(L, dtype):
    """Mamba in_proj: z | xBC stored in the model dtype, dt = softplus(acc + bias)
    routed to an fp32 side output."""
    torch.manual_seed(3)
    m, k = 200, 192
    nmain, ntail = 256 + 64, 24
    n = nmain + ntail
    x = torch.randn(m, k, device=_dev()).to(dtype)
    w = (torch.randn(n, k, device=_dev()) * 0.1).to(dtype)
    bias = torch.randn(ntail, device=_dev())
    out = torch.empty(m, nmain, device=_dev(), dtype=dtype)
    dt = torch.empty(m, ntail, device=_dev())
    L.gemm(x, w, out, act=L.ACT_SOFTPLUS, act_begin=nmain, act_end=n, bias=bias, out2=dt, tail_begin=nmain)
    acc = _gemm_ref(x, w)
    assert rel_l2(out.float(), acc[:, :nmain]) < TOL[dtype]
    assert rel_l2(dt, F.softplus(acc[:, nmain:] + bias)) < (1e-5 if dtype == torch.float32 else 1e-3)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gemm_all_tail(L, dtype):
    """A GEMM whose whole output is the fp32 tail (tail_begin 0): the planner
    may give the scan's dt projection a kernel of its own."""
    torch.manual_seed(4)
    m, k, n = 300, 256, 32
    x = torch.randn(m, k, device=_dev()).to(dtype)
    w = (torch.randn(n, k, device=_dev()) * 0.1).to(dtype)
    bias = torch.randn(n, device=_dev())
    dummy = torch.zeros(m, 8, device=_dev(), dtype=dtype)
    dt = torch.empty(m, n, device=_dev())
    L.gemm(x, w, dummy, act=L.ACT_SOFTPLUS, act_begin=0, act_end=n, bias=bias, out2=dt, tail_begin=0)
    acc = _gemm_ref(x, w)
    assert rel_l2(dt, F.softplus(acc + bias)) < (1e-5 if dtype == torch.float32 else 1e-3)
    assert torch.count_nonzero(dummy) == 0  # nothing written to the main output


def _rope_ref(x, cos, sin, hd, seq):
    t = x.shape[0]
    pos = torch.arange(t, device=x.device) % seq
    c, s = cos[pos], sin[pos]
    xh = x.reshape(t, -1, hd)
    rot = torch.cat((-xh[..., hd // 2:], xh[..., : hd // 2]), -1)
    return (xh * c[:, None, :] + rot * s[:, None, :]).reshape(t, -1)


@pytest.mark.parametrize("dtype,hd", [(torch.bfloat16, 128), (torch.bfloat16, 64), (torch.float32, 64)])
def test_gemm_rope(L, dtype, hd):
    torch.manual_seed(4)
    seq, b, k = 96, 3, 256
    m = seq * b
    nq, nk, nv = 4 * hd, 2 * hd, 2 * hd
    n = nq + nk + nv
    x = torch.randn(m, k, device=_dev()).to(dtype)
    w = (torch.randn(n, k, device=_dev()) * 0.05).to(dtype)
    inv = 1.0 / (10000.0 ** (torch.arange(0, hd, 2, device=_dev()).float() / hd))
    fr = torch.outer(torch.arange(seq, device=_dev()).float(), inv)
    emb = torch.cat((fr, fr), -1)
    cos, sin = emb.cos().contiguous(), emb.sin().contiguous()
    out = torch.empty(m, n, device=_dev(), dtype=dtype)
    L.gemm(x, w, out, rope_cos=cos, rope_sin=sin, rope_begin=0, rope_end=nq + nk, rope_head_dim=hd)
    acc = _gemm_ref(x, w)
    ref = torch.cat((_rope_ref(acc[:, : nq + nk], cos, sin, hd, seq), acc[:, nq + nk:]), -1)
    assert rel_l2(out.float(), ref) < TOL[dtype]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gemm_swiglu(L, dtype):
    torch.manual_seed(5)
    m, k, f = 300, 256, 384
    x = torch.randn(m, k, device=_dev()).to(dtype)
    wg = torch.randn(f, k, device=_dev()) * 0.05
    wu = torch.randn(f, k, device=_dev()) * 0.05
    # interleave in blocks of 64: [g0..63 | u0..63 | g64..127 | u64..127 | ...]
    w = torch.stack((wg.reshape(f // 64, 64, k), wu.reshape(f // 64, 64, k)), 1).reshape(2 * f, k).to(dtype)
    out = torch.empty(m, f, device=_dev(), dtype=dtype)
    L.gemm(x, w, out, swiglu=True)
    xf = x.float()
    ref = F.silu(xf @ wg.to(dtype).float().t()) * (xf @ wu.to(dtype).float().t())
    assert rel_l2(out.float(), ref) < TOL[dtype]


@pytest.mark.parametrize("case", ["plain", "residual", "tail", "swiglu", "rope"])
@pytest.mark.parametrize("m", [4000, 8192])
def test_gemm_pair_tiles(L, case, m):
    """Shapes that take the CTA-pair kernel at its 128-, 192- and 256-column
    widths (on 148 SMs), with a ragged last row tile (m = 4000) that leaves
    the odd CTA of the last pair partly or wholly past the end."""
    torch.manual_seed(6)
    dt = torch.bfloat16
    k = 512
    if case == "swiglu":
        f = 2048
        x = torch.randn(m, k, device=_dev()).to(dt)
        wg, wu = torch.randn(f, k, device=_dev()) * 0.05, torch.randn(f, k, device=_dev()) * 0.05
        w = torch.stack((wg.reshape(f // 64, 64, k), wu.reshape(f // 64, 64, k)), 1).reshape(2 * f, k).to(dt)
        out = torch.empty(m, f, device=_dev(), dtype=dt)
        L.gemm(x, w, out, swiglu=True)
        ref = F.silu(x.float() @ wg.to(dt).float().t()) * (x.float() @ wu.to(dt).float().t())
        assert rel_l2(out.float(), ref) < TOL[dt]
        return
    n = {"plain": 640, "residual": 768, "tail": 3352, "rope": 6144}[case]
    x = torch.randn(m, k, device=_dev()).to(dt)
    w = (torch.randn(n, k, device=_dev()) * 0.05).to(dt)
    acc = _gemm_ref(x, w)
    if case == "plain":
        out = torch.empty(m, n, device=_dev(), dtype=dt)
        L.gemm(x, w, out)
        ref = acc
    elif case == "residual":
        res = torch.randn(m, n, device=_dev()).to(dt)
        parts = L.rowstat(x).reshape(m, 1)
        out = torch.empty(m, n, device=_dev(), dtype=dt)
        L.gemm(x, w, out, rs_parts=parts, rs_inv_k=1.0 / k, rs_eps=1e-6, residual=res)
        r = torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6)
        ref = acc * r + res.float()
    elif case == "tail":
        nmain = n - 24
        bias = torch.randn(24, device=_dev())
        out = torch.empty(m, nmain, device=_dev(), dtype=dt)
        dtail = torch.empty(m, 24, device=_dev())
        L.gemm(x, w, out, act=L.ACT_SOFTPLUS, act_begin=nmain, act_end=n, bias=bias, out2=dtail, tail_begin=nmain)
        assert rel_l2(dtail, F.softplus(acc[:, nmain:] + bias)) < 1e-3
        ref = acc[:, :nmain]
    else:
        hd, seq = 128, m // 2
        inv = 1.0 / (10000.0 ** (torch.arange(0, hd, 2, device=_dev()).float() / hd))
        fr = torch.outer(torch.arange(seq, device=_dev()).float(), inv)
        emb = torch.cat((fr, fr), -1)
        cos, sin = emb.cos().contiguous(), emb.sin().contiguous()
        out = torch.empty(m, n, device=_dev(), dtype=dt)
        rope_end = n - 1024
        L.gemm(x, w, out, rope_cos=cos, rope_sin=sin, rope_begin=0, rope_end=rope_end, rope_head_dim=hd)
        ref = torch.cat((_rope_ref(acc[:, :rope_end], cos, sin, hd, seq), acc[:, rope_end:]), -1)
    torch.cuda.synchronize()
    assert L.device_error() == 0
    assert rel_l2(out.float(), ref) < TOL[dt]


def test_gemm_rejects_bad_alignment(L):
    a = torch.randn(64, 100, device=_dev(), dtype=torch.bfloat16)  # lda=100: 200 B rows, not 16-B multiple
    w = torch.randn(64, 100, device=_dev(), dtype=torch.bfloat16)
    out = torch.empty(64, 64, device=_dev(), dtype=torch.bfloat16)
    with pytest.raises(L.B200KernelError, match="aligned"):
        L.gemm(a, w, out)


# ------------------------------------------------------------ attention
def _attn_ref(q, k, v, b, s, hq, hkv, d, scale, causal):
    q4 = q.float().reshape(b, s, hq, d).transpose(1, 2)
    k4 = k.float().reshape(b, s, hkv, d).transpose(1, 2).repeat_interleave(hq // hkv, 1)
    v4 = v.float().reshape(b, s, hkv, d).transpose(1, 2).repeat_interleave(hq // hkv, 1)
    sc = (q4 @ k4.transpose(-1, -2)) * scale
    if causal:
        sc = sc.masked_fill(torch.triu(torch.ones(s, s, dtype=torch.bool, device=q.device), 1), float("-inf"))
    return (torch.softmax(sc, -1) @ v4).transpose(1, 2).reshape(b * s, hq * d)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("b,s,hq,hkv,d,causal", [(1, 128, 8, 8, 64, False), (2, 100, 4, 2, 64, True),
                                                 (2, 256, 8, 2, 128, True), (1, 70, 2, 1, 32, False),
                                                 # tcgen05 path: several KV blocks, ragged tails, GQA
                                                 (2, 640, 8, 2, 128, True), (1, 1000, 4, 4, 64, False),
                                                 (3, 333, 4, 1, 128, True), (1, 2048, 2, 2, 64, True),
                                                 # 256-row CTAs: second tile partly / wholly past the end
                                                 (1, 300, 4, 2, 128, False), (1, 4096, 4, 1, 128, True)])
def test_attention(L, dtype, b, s, hq, hkv, d, causal):
    torch.manual_seed(6)
    t = b * s
    qkv = torch.randn(t, (hq + 2 * hkv) * d, device=_dev()).to(dtype)
    q, k, v = qkv[:, : hq * d], qkv[:, hq * d: (hq + hkv) * d], qkv[:, (hq + hkv) * d:]
    o = torch.empty(t, hq * d, device=_dev(), dtype=dtype)
    scale = d ** -0.5
    L.attention(q, k, v, o, batch=b, seq=s, hq=hq, hkv=hkv, head_dim=d, scale=scale, causal=causal)
    ref = _attn_ref(q, k, v, b, s, hq, hkv, d, scale, causal)
    assert rel_l2(o.float(), ref) < TOL[dtype]


# --------------------------------------------------------------- conv1d
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("b,s,ch,wd,with_bias,silu", [(3, 150, 1792, 4, False, True),
                                                      # C2 shape: many token tiles per block
                                                      (2, 2048, 1792, 4, False, True),
                                                      # a partial channel block, width 3, bias
                                                      (1, 300, 1000, 3, True, True),
                                                      # width 2, no activation, one row past a tile
                                                      (2, 129, 512, 2, True, False)])
def test_conv1d(L, dtype, b, s, ch, wd, with_bias, silu):
    torch.manual_seed(7)
    src = torch.randn(b * s, ch + 64, device=_dev()).to(dtype)
    x = src[:, 32: 32 + ch]  # strided view, like xBC inside the in_proj output
    w = torch.randn(ch, wd, device=_dev()) * 0.3
    bias = torch.randn(ch, device=_dev()) * 0.1 if with_bias else None
    y = torch.empty(b * s, ch, device=_dev(), dtype=dtype)
    L.conv1d(x, w, y, batch=b, seq=s, act=L.ACT_SILU if silu else L.ACT_NONE, bias=bias)
    xt = x.float().reshape(b, s, ch).transpose(1, 2)
    ref = F.conv1d(F.pad(xt, (wd - 1, 0)), w.unsqueeze(1), bias=bias, groups=ch)
    ref = (F.silu(ref) if silu else ref).transpose(1, 2).reshape(b * s, ch)
    assert rel_l2(y.float(), ref) < TOL[dtype]
    assert L.device_error() == 0


# ------------------------------------------------------------------ ssd
def _ssd_recurrence(x, dt, A, B, C, D, b, s, h, p, g, n):
    """Direct O(S) recurrence (the definition every SSD form must match)."""
    xr = x.double().reshape(b, s, h, p)
    Br = B.double().reshape(b, s, g, n).repeat_interleave(h // g, 2)
    Cr = C.double().reshape(b, s, g, n).repeat_interleave(h // g, 2)
    dtr = dt.double().reshape(b, s, h)
    st = torch.zeros(b, h, p, n, dtype=torch.float64, device=x.device)
    ys = []
    for t in range(s):
        dec = torch.exp(dtr[:, t] * A.double()).reshape(b, h, 1, 1)
        st = dec * st + (dtr[:, t].reshape(b, h, 1, 1) * xr[:, t].unsqueeze(-1) * Br[:, t].unsqueeze(-2))
        ys.append((st * Cr[:, t].unsqueeze(-2)).sum(-1) + D.double().reshape(1, h, 1) * xr[:, t])
    return torch.stack(ys, 1).reshape(b * s, h * p)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("b,s,h,p,g,n,chunk", [(2, 200, 4, 32, 1, 16, 64), (1, 256, 2, 64, 2, 128, 128),
                                               (1, 300, 3, 16, 3, 32, 256),
                                               # tcgen05 scan path: head_dim 64, chunk 256 (full and ragged chunks)
                                               (2, 512, 4, 64, 1, 128, 256), (1, 700, 4, 64, 2, 64, 256),
                                               (3, 300, 2, 64, 1, 128, 256),
                                               # tcgen05 chunk-state + multi-head scan: state 128; head sets,
                                               # two groups, a chunk shorter than 128 rows, many chunks
                                               (2, 1024, 24, 64, 1, 128, 256), (1, 600, 8, 64, 2, 128, 256),
                                               (1, 100, 4, 64, 1, 128, 256), (1, 4096, 2, 64, 1, 128, 256),
                                               # the same path at state 64 and 256 (chunk-parallel states + pass;
                                               # 256: B in two halves, single-buffered x | S_in)
                                               (2, 1024, 24, 64, 1, 64, 256), (2, 512, 6, 64, 3, 64, 256),
                                               (1, 600, 8, 64, 2, 256, 256), (1, 100, 4, 64, 1, 256, 256),
                                               (1, 2048, 4, 64, 1, 256, 256)])
def test_ssd_matches_recurrence(L, dtype, b, s, h, p, g, n, chunk):
    torch.manual_seed(8)
    t = b * s
    x = torch.randn(t, h * p, device=_dev()).to(dtype)
    B = torch.randn(t, g * n, device=_dev()).to(dtype)
    C = torch.randn(t, g * n, device=_dev()).to(dtype)
    dt = torch.rand(t, h, device=_dev()) * 0.099 + 0.001
    A = -torch.exp(torch.rand(h, device=_dev()) * math.log(16))
    D = torch.rand(h, device=_dev())
    z = torch.randn(t, h * p, device=_dev()).to(dtype)
    out = torch.empty(t, h * p, device=_dev(), dtype=dtype)
    gss = torch.empty(t, h, device=_dev())
    L.ssd(x, dt, A, B, C, out, batch=b, seq=s, heads=h, head_dim=p, ngroups=g, state_dim=n, chunk=chunk, D=D, z=z, gss=gss)
    y = _ssd_recurrence(x, dt, A, B, C, D, b, s, h, p, g, n)
    ref = y * F.silu(z.double())
    assert rel_l2(out.float(), ref) < TOL[dtype]
    assert rel_l2(gss, out.float().pow(2).reshape(t, h, p).sum(-1)) < 1e-5


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("gate", [False, True])
@pytest.mark.parametrize("n", [64, 128, 256])
def test_ssd_chunk_path_optional_operands(L, dtype, gate, n):
    """The tcgen05 chunk path with and without z, D and gss."""
    torch.manual_seed(11)
    b, s, h, p, g = 2, 640, 6, 64, 1
    t = b * s
    x = torch.randn(t, h * p, device=_dev()).to(dtype)
    B = torch.randn(t, g * n, device=_dev()).to(dtype)
    C = torch.randn(t, g * n, device=_dev()).to(dtype)
    dt = torch.rand(t, h, device=_dev()) * 0.099 + 0.001
    A = -torch.exp(torch.rand(h, device=_dev()) * math.log(16))
    D = torch.rand(h, device=_dev()) if gate else None
    z = torch.randn(t, h * p, device=_dev()).to(dtype) if gate else None
    out = torch.empty(t, h * p, device=_dev(), dtype=dtype)
    L.ssd(x, dt, A, B, C, out, batch=b, seq=s, heads=h, head_dim=p, ngroups=g, state_dim=n, chunk=256, D=D, z=z)
    y = _ssd_recurrence(x, dt, A, B, C, D if gate else torch.zeros(h, device=_dev()), b, s, h, p, g, n)
    ref = y * F.silu(z.double()) if gate else y
    assert rel_l2(out.float(), ref) < TOL[dtype]
    assert L.device_error() == 0


# ------------------------------------------------------------ embedding
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_embedding(L, dtype):
    torch.manual_seed(9)
    table = torch.randn(1000, 256, device=_dev()).to(dtype)
    ids = torch.randint(0, 1000, (77,), device=_dev())
    out = torch.empty(77, 256, device=_dev(), dtype=dtype)
    L.embedding(ids, table, out)
    assert torch.equal(out, table[ids])


@pytest.mark.parametrize("n", [64, 128])
def test_ssd_steep_decay(L, n):
    """dt*A down to -8 per step: 32 steps of decay span more than exp(80),
    so the tensor-core scan takes its per-element exponential path for the
    G blocks (the factored form would overflow); still the recurrence."""
    torch.manual_seed(12)
    b, s, h, p, g = 1, 512, 4, 64, 1
    t = b * s
    x = torch.randn(t, h * p, device=_dev()).bfloat16()
    B = torch.randn(t, g * n, device=_dev()).bfloat16()
    C = torch.randn(t, g * n, device=_dev()).bfloat16()
    dt = torch.rand(t, h, device=_dev()) * 0.4 + 0.1
    A = -torch.full((h,), 16.0, device=_dev())
    D = torch.rand(h, device=_dev())
    out = torch.empty(t, h * p, device=_dev(), dtype=torch.bfloat16)
    L.ssd(x, dt, A, B, C, out, batch=b, seq=s, heads=h, head_dim=p, ngroups=g, state_dim=n, chunk=256, D=D)
    ref = _ssd_recurrence(x, dt, A, B, C, D, b, s, h, p, g, n)
    assert rel_l2(out.float(), ref) < 1e-2
    assert L.device_error() == 0


@pytest.mark.parametrize("approx", ["none", "tanh"])
@pytest.mark.parametrize("dtype,m", [(torch.bfloat16, 300), (torch.bfloat16, 100), (torch.float32, 100)])
def test_gemm_gelu(L, dtype, m, approx):
    """GELU activation segment with a bias (an MLP's first projection), both
    forms of torch's gelu, on the pair kernel (m > 128), the single-CTA kernel
    and the fp32 path."""
    torch.manual_seed(4)
    k, n = 256, 512
    x = torch.randn(m, k, device=_dev()).to(dtype)
    w = (torch.randn(n, k, device=_dev()) * 0.1).to(dtype)
    bias = torch.randn(n, device=_dev()) * 0.1
    out = torch.empty(m, n, device=_dev(), dtype=dtype)
    code = L.ACT_GELU if approx == "none" else L.ACT_GELU_TANH
    L.gemm(x, w, out, act=code, act_begin=0, act_end=n, bias=bias)
    ref = F.gelu(_gemm_ref(x, w) + bias, approximate=approx)
    assert rel_l2(out.float(), ref) < TOL[dtype]


@pytest.mark.parametrize("dtype,m", [(torch.bfloat16, 300), (torch.float32, 100)])
def test_gemm_bias_only(L, dtype, m):
    """A Linear's bias without an activation (act NONE with a bias on a column range)."""
    torch.manual_seed(5)
    k, n = 192, 256
    x = torch.randn(m, k, device=_dev()).to(dtype)
    w = (torch.randn(n, k, device=_dev()) * 0.1).to(dtype)
    bias = torch.randn(n, device=_dev())
    out = torch.empty(m, n, device=_dev(), dtype=dtype)
    L.gemm(x, w, out, act=L.ACT_NONE, act_begin=0, act_end=n, bias=bias)
    assert rel_l2(out.float(), _gemm_ref(x, w) + bias) < TOL[dtype]
