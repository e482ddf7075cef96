"""SSD (Mamba-2 state-space duality) scans on the CPU -- test infrastructure.

Three statements of the same operator, all on head-major operands
``x [b,h,s,p]``, ``dA, dt [b,h,s]``, ``B, C [b,h,s,n]``:

* :func:`ssd_recurrence` -- the definition, one token at a time
  (reference tests/test_mamba.py:27-38, ``_recurrence``).
* :func:`ssd_chunked` -- the four-step chunked decomposition of the
  reference model (models/mamba.py:163-223, ``ssd_chunked``), restated with
  explicit cumulative sums instead of prefix-matrix products.
* :func:`ssd_quadratic` -- the attention-like dual
  (models/mamba.py:226-251, ``ssd_quadratic``).
"""

from __future__ import annotations

import torch


def ssd_recurrence(x, dA, dt, B, C):
    """state_t = exp(dA_t) state_{t-1} + dt_t x_t B_t^T ;  y_t = state_t C_t.
    Follows tests/test_mamba.py:27-38 of the reference."""
    b, h, s, p = x.shape
    n = B.shape[-1]
    state = torch.zeros(b, h, p, n, dtype=x.dtype)
    ys = []
    for t in range(s):
        decay = torch.exp(dA[:, :, t]).reshape(b, h, 1, 1)
        upd = dt[:, :, t].reshape(b, h, 1, 1) * x[:, :, t].unsqueeze(-1) * B[:, :, t].unsqueeze(-2)
        state = decay * state + upd
        ys.append((state * C[:, :, t].unsqueeze(-2)).sum(-1))
    return torch.stack(ys, dim=2)


def ssd_chunked(x, dA, dt, B, C, chunk: int):
    """Chunked SSD (models/mamba.py:163-223): in-chunk cumsum, diagonal block
    ((C B^T) o L) X, per-chunk states, inter-chunk recurrence + off-diagonal
    output.  Sequences that are not a multiple of ``chunk`` are zero-padded
    (dt = dA = 0 on padding contributes nothing)."""
    b, h, s, p = x.shape
    n = B.shape[-1]
    pad = (-s) % chunk
    if pad:
        zp = lambda t: torch.nn.functional.pad(t, (0, 0, 0, pad)) if t.dim() == 4 else torch.nn.functional.pad(t, (0, pad))
        x, dA, dt, B, C = zp(x), zp(dA), zp(dt), zp(B), zp(C)
    S = s + pad
    c = S // chunk
    xc = x.reshape(b, h, c, chunk, p)
    Bc = B.reshape(b, h, c, chunk, n)
    Cc = C.reshape(b, h, c, chunk, n)
    dAc = dA.reshape(b, h, c, chunk)
    dtc = dt.reshape(b, h, c, chunk)
    cum = torch.cumsum(dAc, -1)                                    # step 1 (mamba.py:195-197)
    last = cum[..., -1:]
    i = torch.arange(chunk)
    within = (i.unsqueeze(1) >= i.unsqueeze(0))
    diff = (cum.unsqueeze(-1) - cum.unsqueeze(-2)).masked_fill(~within, 0.0)
    decay = torch.exp(diff) * within                               # step 2 (mamba.py:199-206)
    y_diag = ((Cc @ Bc.transpose(-1, -2)) * decay * dtc.unsqueeze(-2)) @ xc
    w = (dtc * torch.exp(last - cum)).unsqueeze(-1)                # step 3 (mamba.py:208-210)
    states = (xc * w).transpose(-1, -2) @ Bc                       # [b,h,c,p,n]
    tot = last.squeeze(-1)                                         # step 4 (mamba.py:212-222)
    carried = torch.zeros_like(states)
    run = torch.zeros(b, h, p, n, dtype=x.dtype)
    for z in range(c):
        carried[:, :, z] = run
        run = torch.exp(tot[:, :, z]).reshape(b, h, 1, 1) * run + states[:, :, z]
    y_off = (Cc @ carried.transpose(-1, -2)) * torch.exp(cum).unsqueeze(-1)
    y = (y_diag + y_off).reshape(b, h, S, p)
    return y[:, :, :s]


def ssd_quadratic(x, dA, dt, B, C):
    """M[i,j] = (C_i.B_j) exp(cumA_i - cumA_j) dt_j for j <= i; y = M x
    (models/mamba.py:226-251)."""
    s = x.shape[2]
    cum = torch.cumsum(dA, -1)
    i = torch.arange(s)
    causal = (i.unsqueeze(1) >= i.unsqueeze(0))
    delta = (cum.unsqueeze(-1) - cum.unsqueeze(-2)).masked_fill(~causal, 0.0)
    m = (C @ B.transpose(-1, -2)) * torch.exp(delta) * causal * dt.unsqueeze(-2)
    return m @ x
