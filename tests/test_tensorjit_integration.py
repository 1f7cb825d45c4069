"""The b200 backend behind tensorjit's own API (``tj.jit`` / ``compile_graph``).

These tests need the reference package importable (installed under
``baseline/_ref``); they skip without it.  ``register()`` performs the four
edits the reference's dispatch needs (``tensorjit/compiler.py:21,24-31,34,61-68``).
"""
import pytest
import torch

tj = pytest.importorskip("tensorjit")

import mlir_gpu_kernel_compiler_b200 as tjb  # noqa: E402
from oracle import fixtures as FX  # noqa: E402
from oracle.plan_oracle import evaluate, normwise_error  # noqa: E402


def _mlp(x, g, w1, b1, w2, b2):
    return x + tj.linear(tj.gelu(tj.linear(tj.layer_norm(x, g), w1, b1)), w2, b2)


def test_register_adds_backend_and_keeps_the_plan():
    import tensorjit.compiler as C
    from tensorjit.ir import DType, TensorType

    tjb.register()
    assert "b200" in C.BACKENDS and C.ROW_FUSION_MAX_N["b200"] == 8192
    assert C.pick_backend("cuda") == "b200" and C.pick_backend("cpu") == "c"
    shapes = [(64, 128), (128,), (256, 128), (256,), (128, 256), (128,)]
    g = tj.trace(_mlp, [TensorType(s, DType.bf16) for s in shapes])
    live = tjb.from_tensorjit(C.lower(g, "b200"))
    fixture = FX.load_plan("cuda_mlp__bf16")
    assert [k.kind for k in live.kernels] == [k.kind for k in fixture.kernels]
    assert [[n.op for n in k.nodes] for k in live.kernels] == [[n.op for n in k.nodes] for k in fixture.kernels]
    assert live.to_dict()["kernels"] == fixture.to_dict()["kernels"]


def test_register_reaches_the_torch_compile_backend():
    """torch_backend.py:22 imports compile_graph / pick_backend by name; register() rebinds
    those names too, so torch.compile(..., backend=tj.torch_compile_backend) picks b200."""
    import tensorjit.frontend.torch_backend as TB

    tjb.register()
    assert TB.pick_backend("cuda") == "b200" and TB.pick_backend("cpu") == "c"
    assert TB.compile_graph is tj.compile_graph
    import tensorjit.compiler as C

    assert TB.compile_graph is C.compile_graph and tj.pick_backend is C.pick_backend


@pytest.mark.gpu
def test_torch_compile_on_cuda_runs_b200(monkeypatch):
    """tests/test_mlir_and_torch.py:71-80 of the reference, on CUDA tensors: the FX graph
    goes through torch_compile_backend -> pick_backend -> compile_graph -> b200."""
    import torch.nn.functional as F

    monkeypatch.setenv("TENSORJIT_STRICT", "1")
    tjb.register()
    torch._dynamo.reset()

    class Block(torch.nn.Module):
        def __init__(self, d=32, h=64):
            super().__init__()
            self.ln = torch.nn.LayerNorm(d)
            self.fc1 = torch.nn.Linear(d, h)
            self.fc2 = torch.nn.Linear(h, d)

        def forward(self, x):
            h = F.gelu(self.fc1(self.ln(x)))
            y = x + self.fc2(h)
            return torch.softmax(y, dim=-1) * 2 + y.mean(dim=-1, keepdim=True)

    torch.manual_seed(0)
    m = Block().cuda().eval()
    x = torch.randn(16, 32, device="cuda")
    seen = []
    orig = tjb.compile_program

    def spy(program, **kw):
        cp = orig(program, **kw)
        seen.append(cp)
        return cp

    monkeypatch.setattr(tjb, "compile_program", spy)
    import mlir_gpu_kernel_compiler_b200 as pkg

    monkeypatch.setattr(pkg, "compile_program", spy)
    c = torch.compile(m, backend=tj.torch_compile_backend)
    with torch.no_grad():
        y = c(x)
        ref = m(x)
    assert seen and all(isinstance(cp, tjb.B200Program) for cp in seen)
    torch.testing.assert_close(y, ref, atol=1e-4, rtol=1e-4)


@pytest.mark.gpu
def test_jit_on_cuda_tensors_runs_b200():
    tjb.register()
    torch.manual_seed(0)
    dev = "cuda"
    x, g = torch.randn(64, 128, device=dev), torch.ones(128, device=dev)
    w1, b1 = torch.randn(256, 128, device=dev), torch.randn(256, device=dev)
    w2, b2 = torch.randn(128, 256, device=dev), torch.randn(128, device=dev)
    f = tj.jit(_mlp)                              # no backend: cuda tensors pick "b200"
    out = f(x, g, w1, b1, w2, b2)
    cp = f.compiled(x, g, w1, b1, w2, b2)
    assert isinstance(cp, tjb.B200Program) and cp.num_kernels == 3
    import torch.nn.functional as F

    ref = x + F.linear(F.gelu(F.linear(F.layer_norm(x, (128,), g), w1, b1)), w2, b2)
    assert normwise_error(out, ref) <= 1e-4
    out2 = f(x + 1, g, w1, b1, w2, b2)
    ref2 = (x + 1) + F.linear(F.gelu(F.linear(F.layer_norm(x + 1, (128,), g), w1, b1)), w2, b2)
    assert normwise_error(out2, ref2) <= 1e-4
    assert f.stats.compiles == 1 and f.stats.hits >= 2
