"""Operator vocabulary of the OpGraph.

The raw graph uses the reference's literal vocabulary
(src/torch_helion/capture/ops.py:22-53): layout ops, elementwise binary /
unary ops, last-axis reductions and scans, and the matrix products.  The
B200 canonical form adds the macro ops the sm_100a kernels implement
directly instead of the reference's Loom-only decompositions:

``rope``            RoPE on a token-major [T, H*d] tensor (no W@R GEMM)
``attention``       flash attention with ``causal`` and grouped KV heads
``ssd``             the Mamba-2 chunked scan incl. D-skip and silu(z) gate
``causal_conv1d``   depthwise causal conv over the sequence (+ activation)
``rmsnorm``         a terminal RMSNorm (one not folded into a GEMM)
``embedding``       a row gather
"""

from __future__ import annotations

LAYOUT_OPS = frozenset({"view", "permute", "expand", "clone", "slice", "cat", "cast"})
BINARY_OPS = frozenset({"add", "sub", "mul", "div", "max", "powf"})
UNARY_OPS = frozenset({"exp", "log", "neg", "rsqrt", "sigmoid", "silu", "tanh", "square", "sqrt", "log1p", "softplus",
                       "erf", "gelu"})
REDUCE_OPS = frozenset({"row_sum", "row_max", "row_mean", "row_sumsq"})
SCAN_OPS = frozenset({"row_cumsum"})
MACRO_OPS = frozenset({"rmsnorm", "rope", "rotate_half", "attention", "softmax", "ssd", "causal_conv1d", "embedding"})
ANCHOR_OPS = frozenset({"matmul", "batch_matmul", "attention", "ssd", "causal_conv1d", "rmsnorm", "embedding"})
ELEMENTWISE_OPS = BINARY_OPS | UNARY_OPS

# Ops a B200 GEMM epilogue executes (th_gemm stages); see torch_helion.b200.lower.
EPILOGUE_OPS = frozenset({"add", "mul", "softplus", "silu", "gelu", "rope", "broadcast", "powf", "row_sumsq"})


def is_elementwise(op: str) -> bool:
    return op in ELEMENTWISE_OPS
