"""Pin the CPU oracle (and the workload builders) to the reference.

Golden fixtures come from the reference's own modules
(tests/golden/make_golden.py); the SSD identities are the reference's
known-answer tests (its tests/test_mamba.py:27-74).
"""

from __future__ import annotations

from pathlib import Path

import pytest
import torch

from oracle import models as O
from oracle.ssd import ssd_chunked, ssd_quadratic, ssd_recurrence

G = Path(__file__).resolve().parent / "golden"


def _load(name):
    return torch.load(G / name, weights_only=False)


def test_llama_small_matches_reference():
    d = _load("llama_small_fp32.pt")
    c = d["config"]
    y = O.llama_block_forward(d["state_dict"], d["x"], heads=c["heads"], eps=c["eps"])
    assert O.max_rel_err(y, d["y"]) < 1e-5


@pytest.mark.parametrize("name", ["mamba_small_chunked.pt", "mamba_small_quadratic.pt"])
def test_mamba_small_matches_reference(name):
    d = _load(name)
    c = dict(d["config"])
    y = O.mamba_forward(d["state_dict"], d["u"], n_layers=c["n_layers"], d_model=c["d_model"], expand=c["expand"],
                        headdim=c["headdim"], d_state=c["d_state"], ngroups=c.get("ngroups"), chunk=c["chunk"],
                        use_conv=c.get("use_conv", False), mode=c["mode"])
    assert O.max_rel_err(y, d["y"]) < 1e-5


def test_ssd_forms_match_reference_and_recurrence():
    d = _load("ssd_known_answer.pt")
    ref_rec = ssd_recurrence(d["x"].double(), d["dA"].double(), d["dt"].double(), d["B"].double(), d["C"].double())
    for got in (ssd_chunked(d["x"], d["dA"], d["dt"], d["B"], d["C"], d["chunk"]),
                ssd_quadratic(d["x"], d["dA"], d["dt"], d["B"], d["C"])):
        assert O.max_rel_err(got, d["y_chunked"]) < 1e-5
        assert O.max_rel_err(got, d["y_quadratic"]) < 1e-5
        assert O.max_rel_err(got, ref_rec) < 1e-5


@pytest.mark.parametrize("chunk", [1, 5, 7, 24, 64])
def test_ssd_chunked_any_chunk_and_ragged_length(chunk):
    d = _load("ssd_known_answer.pt")
    ref = ssd_recurrence(d["x"].double(), d["dA"].double(), d["dt"].double(), d["B"].double(), d["C"].double())
    got = ssd_chunked(d["x"].double(), d["dA"].double(), d["dt"].double(), d["B"].double(), d["C"].double(), chunk)
    assert O.max_rel_err(got, ref) < 1e-10


def _check_samples(sd, ref_samples):
    for k, ref in ref_samples.items():
        f = sd[k].detach().double().reshape(-1)
        got = torch.cat((f[:16], torch.tensor([f.sum().item(), f.abs().sum().item()], dtype=torch.float64)))
        assert torch.equal(got[:16], ref[:16]), k
        assert torch.allclose(got[16:], ref[16:], rtol=1e-12, atol=1e-9), k


def test_c1_builder_and_oracle_match_reference():
    from workloads.llama_block import LlamaBlockConfig, build_llama_block

    d = _load("c1_llama.pt")
    cfg = LlamaBlockConfig(batch=1, seq=128, hidden=512, heads=8, intermediate=1408, eps=1e-6, dtype=torch.float32)
    blk = build_llama_block(cfg, seed=0)
    _check_samples(blk.state_dict(), d["weights"])
    x = blk.example_inputs(seed=1)[0]
    assert torch.equal(x, d["x"])
    y = O.llama_block_forward(blk.state_dict(), x, heads=8, eps=1e-6)
    assert O.max_rel_err(y, d["y"]) < 1e-5
    with torch.no_grad():
        assert O.max_rel_err(blk(x), d["y"]) < 1e-6  # the workload module itself


def test_c2_builder_and_oracle_match_reference():
    from workloads import configs

    d = _load("c2_mamba.pt")
    cfg = configs.c2_mamba_block_bf16()
    model = configs.build(cfg, seed=0)
    sd = {k: v for k, v in model.state_dict().items() if "mask" not in k}
    _check_samples(sd, d["weights"])
    u = configs.inputs(model)[0]
    assert torch.allclose(torch.tensor([u.double().sum().item(), u.double().abs().sum().item()], dtype=torch.float64),
                          d["u_stats"].double(), rtol=1e-12)
    y = O.mamba_forward(sd, u, n_layers=1, d_model=768, headdim=64, d_state=128, ngroups=1, chunk=256, use_conv=True)
    sel = y[:, ::97, ::13]
    assert O.rel_l2(sel, d["y_sel"]) < 1e-5
    stats = torch.tensor([y.double().sum().item(), y.double().abs().sum().item(), y.double().pow(2).sum().item()],
                         dtype=torch.float64)
    assert torch.allclose(stats[1:], d["y_stats"][1:].double(), rtol=1e-4)


def test_causal_gqa_extensions_reduce_to_reference():
    """kv_heads == heads and causal=False is exactly the reference block; the
    causal mask equals an explicit masked softmax."""
    d = _load("llama_small_fp32.pt")
    c = d["config"]
    base = O.llama_block_forward(d["state_dict"], d["x"], heads=c["heads"], eps=c["eps"])
    same = O.llama_block_forward(d["state_dict"], d["x"], heads=c["heads"], kv_heads=c["heads"], eps=c["eps"], causal=False)
    assert torch.equal(base, same)
    # causal: only the first token's attention is unchanged (it sees itself only in both forms when s=1)
    caus = O.llama_block_forward(d["state_dict"], d["x"], heads=c["heads"], eps=c["eps"], causal=True)
    assert not torch.allclose(caus, base)
    x1 = d["x"][:, :1]
    one = O.llama_block_forward(d["state_dict"], x1, heads=c["heads"], eps=c["eps"], causal=True)
    assert torch.allclose(one, caus[:, :1], atol=1e-6)
