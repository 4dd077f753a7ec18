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


@pytest.mark.parametrize("low,high", [(-4, 5), (-9, -1)])  # the second: the cut at a negative value
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_ties_at_the_cut_are_kept_in_index_order(low, high, dtype):
    # coarse logits: thousands of exact ties, so the cut falls inside a tie group
    g = torch.Generator().manual_seed(3)
    logits = torch.randint(low, high, (32, 20000), generator=g).to(dtype).to(DEV)
    for seed, (temperature, top_p) in enumerate(((1.0, 0.3), (1.0, 0.6), (1.0, 0.9), (1.3, 0.5))):
        got = _check(logits, temperature, top_p, seed=seed)
        radix = ops.sample_top_p(logits, temperature, top_p, torch.Generator(device=DEV).manual_seed(seed),
                                 force_radix=True).cpu()
        assert torch.equal(got, radix)


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


def _both_paths(logits, temperature, top_p, seed=0):
    fast = ops.sample_top_p(logits, temperature, top_p, torch.Generator(device=DEV).manual_seed(seed))
    radix = ops.sample_top_p(logits, temperature, top_p, torch.Generator(device=DEV).manual_seed(seed),
                             force_radix=True)
    return fast, radix


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("kind", ["normal", "coarse", "flat", "masked", "peaked"])
def test_count_path_equals_radix_path(dtype, kind):
    """The count paths (per 16-bit pattern; for fp32 per value bin, with the cut's
    bin sorted) and the radix-select path use the same fixed-point masses, cut
    and target, so every row gives the same token -- near-ties included, no
    margin. For fp32 the coarse (thousands of ties per value) and flat rows
    overflow the bin buffer and take the radix path inside the kernel."""
    g = torch.Generator().manual_seed(21)
    vocab = 151936
    if kind == "normal":
        x = torch.randn(32, vocab, generator=g) * 4
    elif kind == "coarse":  # thousands of exact ties: the cut falls inside a tie group
        x = torch.randint(-4, 5, (32, vocab), generator=g).float()
    elif kind == "flat":
        x = torch.zeros(32, vocab)
    elif kind == "masked":  # a padded vocabulary: -inf tail
        x = torch.randn(32, vocab, generator=g) * 2
        x[:, 150000:] = float("-inf")
    else:  # one dominant token
        x = torch.randn(32, vocab, generator=g)
        x[torch.arange(32), torch.randint(0, vocab, (32,), generator=g)] = 30.0
    logits = x.to(dtype).to(DEV)
    for seed, (temperature, top_p) in enumerate([(0.7, 0.9), (1.0, 0.5), (1.3, 0.95), (0.8, 1.0), (0.6, 1e-4)]):
        fast, radix = _both_paths(logits, temperature, top_p, seed)
        assert torch.equal(fast, radix), (kind, temperature, top_p, (fast != radix).nonzero()[:4])


@pytest.mark.parametrize("vocab", [7, 1000, 50257])
def test_count_path_equals_radix_path_small_vocab(vocab):
    g = torch.Generator().manual_seed(vocab)
    for dtype in (torch.bfloat16, torch.float16, torch.float32):
        logits = (torch.randn(48, vocab, generator=g) * 3).to(dtype).to(DEV)
        for seed, (temperature, top_p) in enumerate([(0.7, 0.9), (1.0, 1.0), (2.0, 0.3)]):
            fast, radix = _both_paths(logits, temperature, top_p, seed)
            assert torch.equal(fast, radix)


def test_rows_outside_the_count_window_take_the_radix_path():
    g = torch.Generator().manual_seed(4)
    # fp16 at a very high temperature: the massful patterns span more than the window
    logits = (torch.randn(8, 30000, generator=g) * 4).to(torch.float16).to(DEV)
    fast, radix = _both_paths(logits, 1000.0, 0.9, 3)
    assert torch.equal(fast, radix)
    _check(logits, 1000.0, 0.9, seed=3)
    # +inf and all -inf rows next to ordinary ones (each CTA picks its own path)
    x = (torch.randn(4, 5000, generator=g) * 2).to(torch.bfloat16)
    x[1, 123] = float("inf")
    x[2] = float("-inf")
    logits = x.to(DEV)
    fast, radix = _both_paths(logits, 0.9, 0.9, 5)
    assert torch.equal(fast, radix)
    # no finite softmax there (the reference's probabilities are NaN): a valid index, token 0 for all -inf
    assert 0 <= int(fast[1]) < 5000 and int(fast[2]) == 0


def test_fp32_bin_path_ties_and_spans():
    """fp32 rows with a few hundred exact ties near the top (inside one bin),
    rows spanning many binades, rows of tiny values (one bin holds them all:
    the radix path), and temperatures that merge neighbouring values: the
    value-bin path against the radix path."""
    g = torch.Generator().manual_seed(11)
    vocab = 151936
    ties = torch.randn(16, vocab, generator=g) * 2
    ties[:, :400] = 1.25
    wide = torch.randn(16, vocab, generator=g) * 12
    tiny = torch.randn(16, vocab, generator=g) * 1e-3
    for x in (ties, wide, tiny):
        logits = x.to(DEV)
        for seed, (temperature, top_p) in enumerate([(0.7, 0.9), (1.0, 0.5), (3.0, 0.95), (0.5, 0.02)]):
            fast, radix = _both_paths(logits, temperature, top_p, seed)
            assert torch.equal(fast, radix), (temperature, top_p, (fast != radix).nonzero()[:4])
