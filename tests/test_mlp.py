"""A GELU MLP (Linear -> gelu -> Linear) through the whole pipeline: the
capture keeps aten.gelu, the partitioner puts bias + gelu into the first
GEMM's epilogue and the lowering turns it into th_gemm's GELU activation
segment.  CPU: the program's structure and its fp64 interpretation against
the eager module.  GPU: the compiled forward against the eager module in
fp32 on the model's weights (rel-L2 <= 1e-5 fp32, <= 2e-2 bf16)."""

from __future__ import annotations

import pytest
import torch

from conftest import rel_l2


class GeluMLP(torch.nn.Module):
    def __init__(self, d=128, f=512, approx="none", dtype=torch.float32):
        super().__init__()
        torch.manual_seed(0)
        self.up = torch.nn.Linear(d, f).to(dtype)
        self.down = torch.nn.Linear(f, d).to(dtype)
        self.approx = approx

    def forward(self, x):
        return self.down(torch.nn.functional.gelu(self.up(x), approximate=self.approx))


def _compile(tmp_path, approx, dtype, execute):
    from torch_helion import CompileConfig, compile_model

    m = GeluMLP(approx=approx, dtype=dtype).eval()
    x = torch.randn(2, 96, 128, generator=torch.Generator().manual_seed(1)).to(dtype)
    res = compile_model(m, (x,), CompileConfig(run_name="mlp", results_dir=tmp_path, execute=execute))
    return m, x, res


@pytest.mark.parametrize("approx", ["none", "tanh"])
def test_gelu_mlp_program(tmp_path, approx):
    from oracle import interpret as I
    from torch_helion.b200.lower import fp32_outputs, lower_gemm

    m, x, res = _compile(tmp_path, approx, torch.float32, execute=False)
    prog = res.program
    assert [k.kind for k in prog.kernels] == ["gemm", "gemm"]
    plan = lower_gemm(prog.kernels[0], prog.tensors, fp32_outputs(prog))
    assert plan.act == ("gelu" if approx == "none" else "gelu_tanh") and plan.bias is not None
    env = {prog.inputs[0]: x.reshape(prog.tensors[prog.inputs[0]].shape).double()}
    env.update({n: res.graph.params[n].double() for n in prog.params})
    for spec in prog.kernels:
        env.update(I.run_kernel(spec, env))
    with torch.no_grad():
        want = m.double()(x.double())
    assert rel_l2(env[prog.outputs[0]].reshape(want.shape), want) < 1e-12


@pytest.mark.gpu
@pytest.mark.parametrize("approx", ["none", "tanh"])
@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 2e-2)], ids=["fp32", "bf16"])
def test_gelu_mlp_on_gpu(tmp_path, approx, dtype, tol):
    m, x, res = _compile(tmp_path, approx, dtype, execute=True)
    got = res.run(x)[0].float().cpu()
    with torch.no_grad():
        want = GeluMLP(approx=approx, dtype=torch.float32).eval()
        want.load_state_dict({k: v.float() for k, v in m.state_dict().items()})
        ref = want(x.float())
    assert rel_l2(got.reshape(ref.shape), ref) < tol
    assert res.reference_check["ok"], res.reference_check
