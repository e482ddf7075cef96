"""Parity at the BASELINE configurations' own shapes (C3, C4 and every C5
point), on the GPU against the CPU oracle.

Batch rows are independent in both models, so the full-size forward runs on
the GPU through ``compile_model`` and one sequence of its output is compared
with the oracle's batch-1 forward of that sequence (fp32 math on the model's
bf16 weights and inputs, the primary oracle for bf16 configurations).

* C3 -- the Llama-3-8B-geometry block (models/llama_block.py:55-141 with the
  GQA and causal extensions), B8 S4096, and a quicker B1 S1024 case.
* C4 -- the 24-layer Mamba-2 backbone with the token embedding and final
  norm (models/mamba.py:285-359), B16 S2048 vocab 50280.
* C5 -- the standalone chunked scan at batch 8 x 64 heads, chunk 256, every
  (d_state, seqlen) point, through the C ABI (th_ssd), checked on a subset of
  (sequence, head) pairs against the fp64 chunked SSD (models/mamba.py:163-223)
  plus the D skip.  seqlen 16384 is 64 chunks: the longest inter-chunk chain,
  which bounds the drift of the 2-byte state operands of the tensor-core MMAs.

Tolerance: rel-L2 <= 2e-2 (bf16 with fp32 accumulation and fp32 scan state),
the per-kernel bound; the 24-layer C4 backbone, whose bf16 activations between
kernels compound over depth, is held to 3e-2 and to half the error of the
reference's own eager bf16 forward (see the test).
"""

from __future__ import annotations

import pytest
import torch

from conftest import rel_l2
from oracle import models as O
from oracle import ssd as OS

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _compile(model, args, tmp_path):
    from torch_helion import CompileConfig, compile_model

    cfg = CompileConfig(run_name="cfg", results_dir=tmp_path, verify_passes=False, reference_check=False)
    return compile_model(model, args, cfg)


def _sd(model):
    return {k: v.detach() for k, v in model.state_dict().items()}


@pytest.mark.parametrize("batch,seq", [(1, 1024), (8, 4096)], ids=["B1_S1024", "B8_S4096"])
def test_c3_llama8b_block(tmp_path, batch, seq):
    from workloads import configs

    cfg = configs.c3_llama8b_bf16(batch=batch, seq=seq)
    m = configs.build(cfg, seed=0)
    (x,) = m.example_inputs(seed=1)
    res = _compile(m, (x,), tmp_path)
    out = res.run(x)[0]
    got = out[:1].float().cpu()
    del out
    torch.cuda.empty_cache()
    torch.set_num_threads(max(1, torch.get_num_threads()))
    with torch.no_grad():
        ref = O.llama_block_forward(_sd(m), x[:1], heads=cfg.heads, kv_heads=cfg.kv_heads, eps=cfg.eps,
                                    rope_theta=cfg.rope_theta, causal=cfg.causal, model_dtype=cfg.dtype)
    err = rel_l2(got, ref)
    print(f"C3 B{batch} S{seq}: sequence 0 rel-L2 vs oracle {err:.3e}")
    assert err < TOL
    kinds = [k.kind for k in res.program.kernels]
    assert kinds.count("attention") == 1 and set(kinds) == {"gemm", "attention"}, kinds


def test_c4_mamba24_backbone(tmp_path):
    from workloads import configs

    cfg = configs.c4_mamba24_bf16()
    m = configs.build(cfg, seed=0)
    (ids,) = m.example_inputs(seed=1)
    res = _compile(m, (ids,), tmp_path)
    out = res.run(ids)[0]
    assert tuple(out.shape) == (16, 2048, 1024)
    got = out[:1].float().cpu()
    last = out[-1:].float().cpu()
    del out
    with torch.no_grad():
        sd = _sd(m)
        kw = dict(n_layers=cfg.n_layers, d_model=cfg.d_model, expand=cfg.expand, headdim=cfg.headdim,
                  d_state=cfg.d_state, ngroups=cfg.ngroups, chunk=cfg.chunk, eps=cfg.eps, use_conv=cfg.use_conv,
                  d_conv=cfg.d_conv, mode=cfg.mode, embedding=True, lm_head=cfg.tie_lm_head)
        ref = O.mamba_forward(sd, ids[:1], **kw)
        ref_last = O.mamba_forward(sd, ids[-1:], **kw)
        eager_bf16 = m(ids[:1]).float()  # the reference's own eager forward in the model dtype
    err, err_last = rel_l2(got, ref), rel_l2(last, ref_last)
    err_eager = rel_l2(eager_bf16, ref)
    print(f"C4 B16 S2048 24 layers: sequence 0 rel-L2 {err:.3e}, sequence 15 rel-L2 {err_last:.3e}; "
          f"the eager bf16 forward itself: {err_eager:.3e}")
    # 2e-2 is the per-kernel bound (each kernel is held to it at the C2 and C5 shapes).  Through 24 layers
    # with bf16 activations between kernels the roundings compound: rounding only the residual stream to
    # bf16 after every layer, with everything else in fp32, already costs 1.45e-2 here, and the
    # reference's own eager bf16 forward lands at about 8e-2.  The model-level bound is therefore 3e-2
    # and at most half of the eager bf16 forward's own error.
    assert err < 3e-2 and err_last < 3e-2
    assert err < 0.5 * err_eager
    kinds = [k.kind for k in res.program.kernels]
    assert kinds.count("ssd") == 24 and kinds[0] == "embedding" and kinds[-1] == "rmsnorm"


def _c5_oracle(t, b, s, h_idx, p, n):
    """fp64 chunked SSD + D skip for sequence b and heads h_idx: [s, len(h_idx), p]."""
    H = t["A"].numel()
    rows = slice(b * s, (b + 1) * s)
    x = t["x"][rows].double().reshape(s, H, p)[:, h_idx].permute(1, 0, 2).unsqueeze(0)
    dt = t["dt"][rows].double()[:, h_idx].t().unsqueeze(0)
    A = t["A"].double()[h_idx]
    B = t["B"][rows].double().reshape(1, 1, s, n).expand(1, len(h_idx), s, n)
    C = t["C"][rows].double().reshape(1, 1, s, n).expand(1, len(h_idx), s, n)
    y = OS.ssd_chunked(x, dt * A.reshape(1, -1, 1), dt, B, C, 256)
    y = y + x * t["D"].double()[h_idx].reshape(1, -1, 1, 1)
    return y[0].permute(1, 0, 2)


@pytest.mark.parametrize("seq", [512, 2048, 8192, 16384])
@pytest.mark.parametrize("d_state", [64, 128, 256])
def test_c5_ssd_point(d_state, seq):
    from torch_helion.b200 import lib
    from workloads import configs

    g = configs.C5_GRID
    b, H, P = g["batch"], g["nheads"], g["headdim"]
    t = configs.ssd_inputs(b, seq, H, P, d_state, ngroups=1, seed=1)
    dev = {k: v.to("cuda:0") for k, v in t.items()}
    out = torch.empty_like(dev["x"])
    lib.ssd(dev["x"], dev["dt"], dev["A"], dev["B"], dev["C"], out, batch=b, seq=seq, heads=H, head_dim=P, ngroups=1,
            state_dim=d_state, chunk=256, D=dev["D"])
    torch.cuda.synchronize()
    assert lib.device_error() == 0
    y = out.float().cpu()
    del out, dev
    heads = [0, 21, 42, 63]
    for bi in (0, b - 1):
        ref = _c5_oracle(t, bi, seq, heads, P, d_state)
        got = y[bi * seq:(bi + 1) * seq].reshape(seq, H, P)[:, heads].double()
        err = rel_l2(got, ref)
        # the last chunk alone: the end of the longest inter-chunk chain
        tail = rel_l2(got[-256:], ref[-256:])
        print(f"C5 d_state {d_state} seq {seq} sequence {bi}: rel-L2 {err:.3e} (last chunk {tail:.3e})")
        assert err < TOL and tail < TOL
