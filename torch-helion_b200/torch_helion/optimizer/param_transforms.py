"""Offline weight transforms (compile time, never in place).

``fold_gain_into_weight`` is the reference identity (x*g) @ W = x @ (diag(g) W)
(src/torch_helion/optimizer/param_transforms.py:18-20).  The reference's
rotate-half matrices (:23-44) are not needed on B200: RoPE runs in the GEMM
epilogue on paired columns.  ``swiglu_interleave`` lays the gate/up weights
out for th_gemm's SwiGLU epilogue.
"""

from __future__ import annotations

import torch


def fold_gain_into_weight(gain: torch.Tensor, w_kn: torch.Tensor) -> torch.Tensor:
    """``w_kn [K, N]`` scaled row-wise by ``gain [K]`` (fp32 math, cast back)."""
    return (gain.float().reshape(-1, 1) * w_kn.float()).to(w_kn.dtype)


def swiglu_interleave(w_gate_nk: torch.Tensor, w_up_nk: torch.Tensor, block: int = 64) -> torch.Tensor:
    """[F, K] gate and up weights -> [2F, K] in blocks of ``block`` rows:
    [gate 0:64 | up 0:64 | gate 64:128 | up 64:128 | ...]."""
    f, k = w_gate_nk.shape
    if f % block:
        raise ValueError(f"SwiGLU width {f} is not a multiple of {block}")
    g = w_gate_nk.reshape(f // block, block, k)
    u = w_up_nk.reshape(f // block, block, k)
    return torch.stack((g, u), 1).reshape(2 * f, k).contiguous()
