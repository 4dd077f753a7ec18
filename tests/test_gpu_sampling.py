"""Top-p sampling kernel (C ABI pkv_sample_top_p through ops.sample_top_p).

The kernel keeps the reference's nucleus (src/triton_kernels/paged_kv.py:418-450)
and draws with one uniform per row from the caller's generator by the inverse
CDF of the kept tokens in index order. The oracle applies the same rule to the
same uniforms, so tokens must be equal, except on rows where float rounding
decides: the running probability within 1e-6 of top_p at the cut, or the
target within 1e-6 of a CDF step (both reported by the oracle; the kernel's
probabilities are fp32 and their sums fp64, the oracle's fp64). With a
151,936-token vocabulary and a flat distribution each token carries ~1e-5,
so a good share of rows sits that close to a step and is not counted.
"""

from __future__ import annotations

import pytest
import torch

from grpo_training_engine_b200 import ops
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _check(logits, temperature, top_p, seed=0, min_checked=0.3):
    g1 = torch.Generator(device=DEV).manual_seed(seed)
    g2 = torch.Generator(device=DEV).manual_seed(seed)
    got = ops.sample_top_p(logits, temperature, top_p, g1).cpu()
    u = torch.rand(logits.shape[0], device=DEV, dtype=torch.float32, generator=g2)
    ref, cut_margin, draw_margin = oracle.sample_top_p(logits.cpu(), temperature, top_p, u.cpu())
    decided = (cut_margin > 1e-6) & (draw_margin > 1e-6)
    assert decided.mean() >= min_checked, decided.mean()
    mism = (got != ref).numpy() & decided
    assert not mism.any(), (got[mism], ref[mism])
    return got


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("vocab", [151936, 50257, 1000, 7])
@pytest.mark.parametrize("temperature,top_p", [(0.7, 0.9), (1.0, 0.5), (1.3, 0.95), (0.8, 1.0)])
def test_sample_matches_oracle(dtype, vocab, temperature, top_p):
    g = torch.Generator().manual_seed(vocab + int(100 * top_p))
    logits = (torch.randn(24, vocab, generator=g) * 4).to(dtype).to(DEV)
    _check(logits, temperature, top_p, seed=vocab)


def test_ties_at_the_cut_are_kept_in_index_order():
    # coarse logits: thousands of exact ties, so the cut falls inside a tie group
    g = torch.Generator().manual_seed(3)
    logits = torch.randint(-4, 5, (32, 20000), generator=g).to(torch.bfloat16).to(DEV)
    for seed, top_p in enumerate((0.3, 0.6, 0.9)):
        _check(logits, 1.0, top_p, seed=seed)


def test_tiny_top_p_is_argmax_and_strided_rows():
    g = torch.Generator().manual_seed(5)
    wide = (torch.randn(16, 151936 + 64, generator=g) * 3).to(torch.bfloat16).to(DEV)
    logits = wide[:, 32:32 + 151936]  # row stride > vocab
    got = ops.sample_top_p(logits, 0.7, 1e-6, torch.Generator(device=DEV).manual_seed(0))
    assert torch.equal(got, logits.float().argmax(-1))
    _check(logits, 0.7, 0.9, seed=9)


def test_sampling_frequencies_follow_the_nucleus():
    # one small row sampled many times: empirical frequencies ~ renormalised nucleus
    logits = torch.tensor([[2.0, 1.5, 1.0, 0.5, 0.0, -1.0, -3.0, -5.0]], device=DEV).repeat(4096, 1)
    got = ops.sample_top_p(logits, 1.0, 0.8, torch.Generator(device=DEV).manual_seed(1)).cpu()
    p = torch.softmax(logits[0].cpu().double(), 0)
    run = p.cumsum(0)
    keep = run <= 0.8
    keep[0] = True
    q = torch.where(keep, p, torch.zeros_like(p))
    q /= q.sum()
    freq = torch.bincount(got, minlength=8).double() / got.numel()
    assert (freq[~keep] == 0).all()
    assert float((freq - q).abs().max()) < 0.03


def test_invalid_arguments():
    logits = torch.randn(2, 10, device=DEV)
    with pytest.raises(ValueError):
        ops.sample_top_p(logits, 0.0, 0.9)
    with pytest.raises(ValueError):
        ops.sample_top_p(logits, 1.0, 0.0)
    with pytest.raises(ValueError):
        ops.sample_top_p(logits[0], 1.0, 0.9)
