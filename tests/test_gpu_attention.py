"""The fused tcgen05 attention kernel on the GPU.

The fixture parity suite (test_gpu_parity.py) already runs every attention
fixture through the fused kernel against the reference's golden outputs; these
tests add what the fixtures cannot show: the fused and unfused programs agree,
the kernel really is the one that ran, and the online softmax stays exact when
the running row maximum moves (scores that grow along the key axis force the
lazy rescale of the TMEM accumulator on many key blocks), checked against a
plain PyTorch fp32 attention.
"""
import pytest
import torch

from oracle import fixtures as FX
from oracle.plan_oracle import evaluate, normwise_error

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _prog(case, **kw):
    from mlir_gpu_kernel_compiler_b200 import B200Program

    return B200Program(FX.load_plan(case), device="cuda", **kw)


def _resized_attention_plan(b, sq, sk, dtype="bf16"):
    """The reference's plan for softmax(q k^T / 8) v (fixture attention_ragged:
    batch 3, 200 queries, 300 keys) with the batch and sequence lengths replaced."""
    from mlir_gpu_kernel_compiler_b200.plan import PProgram

    d = FX.load_plan("attention_ragged__bf16").to_dict()
    sub = {3: b, 200: sq, 300: sk}
    fix = lambda shape: [sub.get(x, x) for x in shape]  # noqa: E731
    for n in d["nodes"]:
        n["shape"] = fix(n["shape"])
        n["dtype"] = dtype
    for k in d["kernels"]:
        k["iter_shape"] = fix(k["iter_shape"])
        for st in k.get("stages", []):
            st["iter_shape"] = fix(st["iter_shape"])
        if k["kind"] == "row":
            k["rows"], k["n"] = fix(k["rows"]), sk
    d["meta"] = {"dtype": dtype}
    return PProgram.from_dict(d)


def _torch_attention(q, k, v, scale):
    s = torch.matmul(q.float(), k.float().transpose(-1, -2)) * scale
    return torch.matmul(torch.softmax(s, dim=-1), v.float())


@pytest.mark.parametrize("case", ["attention_core__bf16", "attention_ragged__bf16", "attention_ragged__f16",
                                  "attention_short__f16", "attention_heads__bf16"])
def test_fused_matches_unfused(case):
    ins = [t.cuda() for t in FX.case_inputs(case)]
    fused = _prog(case)
    plain = _prog(case, fuse_kernels=False)
    assert any(ks.family == "attention" for ks in fused.kernel_sources)
    assert not any(ks.family == "attention" for ks in plain.kernel_sources)
    assert fused.num_kernels < plain.num_kernels
    yf = fused(*ins)
    yp = plain(*ins)
    torch.cuda.synchronize()
    fused.check()
    plain.check()
    for a, b in zip(yf, yp):
        assert a.shape == b.shape and a.dtype == b.dtype
        assert normwise_error(a, b) <= TOL


@pytest.mark.parametrize("case,scale", [("attention_core__bf16", 0.125), ("attention_ragged__f16", 0.125)])
def test_online_softmax_with_growing_row_max(case, scale):
    """Keys whose norm grows with their position: every key block raises the row max
    by more than the rescale threshold, so O is rescaled in TMEM on most blocks."""
    prog = _prog(case)
    plan = prog.pplan
    q_shape, k_shape, v_shape = (tuple(x.shape) for x in plan.inputs)
    dt = {"bf16": torch.bfloat16, "f16": torch.float16}[plan.inputs[0].dtype]
    g = torch.Generator(device="cuda").manual_seed(7)
    q = (torch.rand(q_shape, generator=g, device="cuda") + 0.5).to(dt)
    sk = k_shape[-2]
    ramp = torch.linspace(0.0, 6.0, sk, device="cuda").view(*([1] * (len(k_shape) - 2)), sk, 1)
    k = ((torch.rand(k_shape, generator=g, device="cuda") + 0.5) * ramp).to(dt)
    v = torch.randn(v_shape, generator=g, device="cuda").to(dt)
    y = prog(q, k, v)[0]
    torch.cuda.synchronize()
    prog.check()
    ref = _torch_attention(q, k, v, scale)
    assert torch.isfinite(y.float()).all()
    assert normwise_error(y, ref) <= TOL


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_online_softmax_rescales_on_every_block_of_a_long_sequence(dtype):
    """2050 keys (17 blocks, the last one 2 keys wide) whose scores grow by more than
    the rescale threshold from block to block, 300 queries (a partial second tile)."""
    from mlir_gpu_kernel_compiler_b200 import B200Program

    b, sq, sk = 2, 300, 2050
    prog = B200Program(_resized_attention_plan(b, sq, sk, dtype), device="cuda")
    assert [ks.family for ks in prog.kernel_sources] == ["attention"]
    dt = {"bf16": torch.bfloat16, "f16": torch.float16}[dtype]
    g = torch.Generator(device="cuda").manual_seed(11)
    q = (torch.rand((b, sq, 64), generator=g, device="cuda") * 0.2 + 0.9).to(dt)
    # score ~ 64 * ramp / 8 grows by ~8.7 (log2 units) per 128-key block
    ramp = torch.linspace(0.0, 12.0, sk, device="cuda").view(1, sk, 1)
    k = ((torch.rand((b, sk, 64), generator=g, device="cuda") * 0.2 + 0.9) * ramp).to(dt)
    v = torch.randn((b, sk, 64), generator=g, device="cuda").to(dt)
    y = prog(q, k, v)[0]
    torch.cuda.synchronize()
    prog.check()
    ref = _torch_attention(q, k, v, 1.0 / 8.0)
    assert torch.isfinite(y.float()).all()
    assert normwise_error(y, ref) <= TOL


def test_graph_replay_with_new_inputs_and_large_scores():
    case = "attention_heads__bf16"
    prog = _prog(case, use_graph=True)
    ins = [t.cuda() for t in FX.case_inputs(case)]
    y1 = prog(*ins)[0].clone()
    ins2 = [ins[0] * 4.0] + ins[1:]        # 16x larger scores: sharper softmax
    y2 = prog(*ins2)[0]
    torch.cuda.synchronize()
    prog.check()
    # against the f32 oracle.  With 4x larger scores the bf16 storage of q/k alone moves
    # the result by about the tolerance, so there the fused program must be no less
    # accurate than the unfused chain (which also rounds the scores to bf16).
    plan = prog.pplan
    plain = _prog(case, fuse_kernels=False)
    ref1 = evaluate(plan, [t.cpu() for t in ins])[0]
    assert normwise_error(y1, ref1) <= TOL
    ref2 = evaluate(plan, [t.cpu() for t in ins2])[0]
    assert normwise_error(y2, ref2) <= normwise_error(plain(*ins2)[0], ref2)
    assert prog.stats["graph_replays"] == 2


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_packed_f32x2_softmax_is_bit_identical(monkeypatch, dtype):
    """The softmax's scale-and-shift FMAs and running sums as packed f32x2 instructions (knob
    F2) round each lane exactly like the scalar code, in the same order: the output must be
    the same bits, here on the long sequence whose row maximum moves on every key block and
    on the head-split fixture."""
    from mlir_gpu_kernel_compiler_b200 import B200Program

    b, sq, sk = 2, 300, 2050
    dt = {"bf16": torch.bfloat16, "f16": torch.float16}[dtype]
    g = torch.Generator(device="cuda").manual_seed(12)
    q = (torch.rand((b, sq, 64), generator=g, device="cuda") * 0.2 + 0.9).to(dt)
    ramp = torch.linspace(0.0, 12.0, sk, device="cuda").view(1, sk, 1)
    k = ((torch.rand((b, sk, 64), generator=g, device="cuda") * 0.2 + 0.9) * ramp).to(dt)
    v = torch.randn((b, sk, 64), generator=g, device="cuda").to(dt)
    heads = [t.cuda() for t in FX.case_inputs("attention_heads__bf16")]
    outs = {}
    for f2 in ("0", "1"):
        monkeypatch.setenv("TENSORJIT_B200_ATTN", f"F2={f2}")
        p1 = B200Program(_resized_attention_plan(b, sq, sk, dtype), device="cuda")
        assert ("F2 = true" in p1.source) == (f2 == "1")
        outs[f2] = [p1(q, k, v)[0]]
        if dtype == "bf16":
            outs[f2].append(_prog("attention_heads__bf16")(*heads)[0])
        torch.cuda.synchronize()
        p1.check()
    for a, c in zip(outs["0"], outs["1"]):
        assert torch.equal(a, c)
