"""pkv_linear (tcgen05 projection GEMM) against an fp32 torch reference.

The shapes are the projections of one decode step of the rollout model
(DeepSeek-R1-Distill-Qwen-1.5B geometry, 128 sequences): stacked q/k/v with
bias (N 2048, K 1536), o_proj (1536, 1536), the stacked gate/up with the SiLU
gate (N 8960, K 1536), down_proj (1536, 8960), the LM head (151,936, 1536),
plus odd row counts, fp16, strided views and rows beyond one 128-row launch.
The reference is x.float() @ W.float().T (+ bias) in fp32, rounded once to the
16-bit dtype; the kernel accumulates in fp32 in another order, so an output
element may land one 16-bit rounding step away from it, and rarely.
"""

from __future__ import annotations

import pytest
import torch

from grpo_training_engine_b200 import ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _operands(seed, rows, n, k, dtype, bias=False, w_rows=None):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(rows, k, device=DEV, generator=g).to(dtype)
    w = (torch.randn(w_rows or n, k, device=DEV, generator=g) / k ** 0.5).to(dtype)
    b = (torch.randn(n, device=DEV, generator=g) * 0.5).to(dtype) if bias else None
    return x, w, b


def _close(out, ref_fp32, dtype):
    """out within one 16-bit rounding step of the fp32 reference, and equal to
    its rounding on nearly every element."""
    ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10
    want = ref_fp32.to(dtype)
    diff = (out.float() - want.float()).abs()
    assert bool((diff <= ref_fp32.abs() * ulp + 1e-4).all()), float((diff - ref_fp32.abs() * ulp).max())
    assert float((out != want).float().mean()) < 0.02


SHAPES = [
    # rows, n, k, bias
    (128, 2048, 1536, True),     # q/k/v stacked, with their biases
    (128, 1536, 1536, False),    # o_proj
    (128, 1536, 8960, False),    # down_proj (split K)
    (128, 151936, 1536, False),  # LM head (256-column tiles, a partial last tile)
    (1, 1536, 1536, False),      # one sequence
    (37, 2048, 1536, True),      # a ragged batch
    (200, 1536, 1536, False),    # two launches of rows
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"r{s[0]}n{s[1]}k{s[2]}{'b' if s[3] else ''}")
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_linear_matches_fp32_reference(shape, dtype):
    rows, n, k, bias = shape
    if dtype == torch.float16 and n > 20000:
        pytest.skip("one LM-head case is enough")
    x, w, b = _operands(rows * 7 + n, rows, n, k, dtype, bias)
    out = ops.linear(x, w, b)
    torch.cuda.synchronize()
    ref = x.float() @ w.float().T
    if b is not None:
        ref = ref + b.float()
    _close(out, ref, dtype)
    # deterministic: split-K partials are added in split order
    again = ops.linear(x, w, b)
    assert torch.equal(out, again)


@pytest.mark.parametrize("rows", [128, 5])
def test_linear_silu_gate_matches_the_mlp_rounding(rows):
    n, k = 8960, 1536
    x, w, _ = _operands(3 + rows, rows, n, k, torch.bfloat16, w_rows=2 * n)
    out = ops.linear(x, w, silu_gate=True)
    torch.cuda.synchronize()
    gate = (x.float() @ w[:n].float().T).to(torch.bfloat16)
    up = (x.float() @ w[n:].float().T).to(torch.bfloat16)
    want = (torch.nn.functional.silu(gate.float()).to(torch.bfloat16).float() * up.float()).to(torch.bfloat16)
    diff = (out.float() - want.float()).abs()
    # a gate or up element one rounding step off moves the product by about as much
    assert bool((diff <= want.float().abs() * 2.0 ** -6 + 2e-3).all()), float(diff.max())
    assert float((out != want).float().mean()) < 0.05
    assert torch.equal(out, ops.linear(x, w, silu_gate=True))
    # the gate_proj and up_proj weights as two tensors (the modules' own): same bits
    gate_w, up_w = w[:n].clone(), w[n:].clone()
    assert torch.equal(out, ops.linear(x, gate_w, silu_gate=True, weight_up=up_w))


def test_linear_strided_views_and_out():
    k, n = 1536, 2048
    big = torch.randn(64, 3 * k, device=DEV).to(torch.bfloat16)
    x = big[:, k:2 * k]  # row stride 3 k
    w = (torch.randn(n, k, device=DEV) / k ** 0.5).to(torch.bfloat16)
    out_big = torch.full((64, n + 64), 7.0, device=DEV, dtype=torch.bfloat16)
    out = out_big[:, 32:32 + n]
    ops.linear(x, w, out=out)
    torch.cuda.synchronize()
    _close(out, x.float() @ w.float().T, torch.bfloat16)
    assert bool((out_big[:, :32] == 7).all()) and bool((out_big[:, 32 + n:] == 7).all())


def test_linear_rejects_what_it_cannot_serve():
    x = torch.randn(4, 100, device=DEV).to(torch.bfloat16)  # K not a multiple of 64
    w = torch.randn(32, 100, device=DEV).to(torch.bfloat16)
    assert not ops.linear_supported(x, w)
    with pytest.raises(ValueError):
        ops.linear(x, w)


@pytest.mark.parametrize("shape", [(128, 2048, 1536, True), (128, 1536, 8960, False), (37, 1536, 1536, False),
                                   (128, 151936, 1536, False)],
                         ids=lambda s: f"r{s[0]}n{s[1]}k{s[2]}{'b' if s[3] else ''}")
def test_linear_static_weights_same_bits(shape):
    """weights_static only moves the first weight tiles before the dependency
    wait: the result is bit-identical."""
    rows, n, k, bias = shape
    x, w, b = _operands(11 + n, rows, n, k, torch.bfloat16, bias)
    plain = ops.linear(x, w, b)
    static = ops.linear(x, w, b, weights_static=True)
    torch.cuda.synchronize()
    assert torch.equal(plain, static)


def test_linear_static_weights_reads_x_after_the_previous_kernel():
    """x is rewritten in place by the kernel just before each launch (and by
    the previous projection in a chain): a launch that read x before its
    dependency wait would see the old values."""
    k, n = 1536, 2048
    g = torch.Generator(device=DEV).manual_seed(5)
    x0 = torch.randn(128, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device=DEV, generator=g) / k ** 0.5).to(torch.bfloat16)
    xbuf = torch.empty_like(x0)
    outs = []
    for i in range(6):
        xbuf.copy_(x0 * (i + 1))  # the previous kernel in the stream writes x
        outs.append(ops.linear(xbuf, w, weights_static=True))
    torch.cuda.synchronize()
    for i, o in enumerate(outs):
        assert torch.equal(o, ops.linear((x0 * (i + 1)).contiguous(), w)), i
    # rmsnorm -> gate/up (SiLU) -> down, each consuming the previous launch's output
    inter = 8960
    gate = (torch.randn(inter, k, device=DEV, generator=g) / k ** 0.5).to(torch.bfloat16)
    up = (torch.randn(inter, k, device=DEV, generator=g) / k ** 0.5).to(torch.bfloat16)
    down = (torch.randn(k, inter, device=DEV, generator=g) / inter ** 0.5).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(k, device=DEV, generator=g)).to(torch.bfloat16)
    res = torch.randn(128, k, device=DEV, generator=g).to(torch.bfloat16)
    chained = []
    for i in range(3):
        h, _ = ops.add_rmsnorm(x0 * (i + 1), nw, 1e-6, residual=res)
        a = ops.linear(h, gate, silu_gate=True, weight_up=up, weights_static=True)
        chained.append(ops.linear(a, down, weights_static=True))
    torch.cuda.synchronize()
    for i, o in enumerate(chained):
        h, _ = ops.add_rmsnorm(x0 * (i + 1), nw, 1e-6, residual=res)
        torch.cuda.synchronize()
        a = ops.linear(h, gate, silu_gate=True, weight_up=up)
        torch.cuda.synchronize()
        assert torch.equal(o, ops.linear(a, down)), i
