"""PKV_DECODE_EARLY_START (paged_attention_decode(early_start=True)).

A step of several layers whose later launches schedule their first unit and
start loading its pages before the previous layer's launch has finished must
give the same outputs and the same cache bytes as the same step launched
without it, eagerly and replayed from a CUDA graph. The cases cover CTAs
without units (few sequences), split sequences merged inside the launch, two
head groups at head_dim 64, RoPE inside the launch, and a batch with enough
units for the schedule's counted tail.
"""

from __future__ import annotations

import hashlib
import math

import pytest
import torch

from conftest import ATOL
from grpo_training_engine_b200 import paged_attention_decode, plan_decode
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"
LAYERS = 3

CASES = [
    # (batch, hq, hkv, head_dim, block_size, ctxs or (lo, hi) for a seeded uniform draw, pages_per_split)
    (4, 12, 2, 128, 16, [1, 16, 17, 777], 0),          # few units: most CTAs get none
    (3, 28, 4, 128, 16, [5000, 33, 2048], 8),           # split-K, merged inside the launch
    (2, 40, 2, 64, 16, [500, 1], 0),                    # two head groups, head_dim 64
    (1024, 12, 2, 128, 16, (16, 160), 0),               # 2048 units: the counted tail of the schedule
]


def _sha(*tensors: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.contiguous().view(torch.uint8).cpu().numpy().tobytes())
    return h.hexdigest()


def _case(seed, batch, hq, hkv, d, bs, ctxs):
    g = torch.Generator().manual_seed(seed)
    if isinstance(ctxs, tuple):
        ctxs = torch.randint(ctxs[0], ctxs[1], (batch,), generator=g).tolist()
    max_blocks = max(math.ceil(c / bs) for c in ctxs) + 1
    num_blocks = batch * max_blocks + 3
    # every sequence owns its pages (the appended token must not land in a page
    # another sequence reads in the same launch)
    bt = torch.randperm(num_blocks, generator=g)[: batch * max_blocks].reshape(batch, max_blocks).int()
    q = torch.randn(LAYERS, batch, hq, d, generator=g).to(torch.bfloat16)
    kn = torch.randn(LAYERS, batch, hkv, d, generator=g).to(torch.bfloat16)
    vn = torch.randn(LAYERS, batch, hkv, d, generator=g).to(torch.bfloat16)
    kc = torch.randn(LAYERS, num_blocks, hkv, bs, d, generator=g).to(torch.bfloat16)
    vc = torch.randn(LAYERS, num_blocks, hkv, bs, d, generator=g).to(torch.bfloat16)
    ctx = torch.tensor(ctxs, dtype=torch.int32)
    return [t.to(DEV) for t in (q, kn, vn, kc, vc, bt, ctx)]


def _step(q, kn, vn, kc, vc, bt, ctx, pps, early, outs, rope=None, status=None):
    """One plan, then every layer's fused append + decode (the layers after the
    first with early start when `early`)."""
    hq, d = q.shape[2], q.shape[3]
    plan = plan_decode(ctx, hq, kc.shape[2], d, kc.shape[3], bt.shape[1], pages_per_split=pps)
    for layer in range(LAYERS):
        paged_attention_decode(q[layer], kc[layer], vc[layer], bt, ctx, out=outs[layer], plan=plan,
                               k_new=kn[layer], v_new=vn[layer], rope=rope, status=status,
                               early_start=early and layer > 0)


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"b{c[0]}q{c[1]}kv{c[2]}d{c[3]}p{c[6]}")
def test_early_start_same_outputs_and_cache(case):
    batch, hq, hkv, d, bs, ctxs, pps = case
    q, kn, vn, kc, vc, bt, ctx = _case(3, batch, hq, hkv, d, bs, ctxs)
    kc0, vc0 = kc.clone(), vc.clone()
    plain = torch.empty(LAYERS, batch, hq, d, device=DEV)
    early = torch.empty_like(plain)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    _step(q, kn, vn, kc, vc, bt, ctx, pps, False, plain)
    kc1, vc1 = kc0.clone(), vc0.clone()
    _step(q, kn, vn, kc1, vc1, bt, ctx, pps, True, early, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(plain, early)
    assert _sha(kc, vc) == _sha(kc1, vc1)
    # and the first layer against the oracle (the appended caches, post-append lengths)
    want = oracle.decode(q[0].cpu(), kc[0].cpu(), vc[0].cpu(), bt.cpu(), ctx.cpu())
    assert float((early[0].cpu() - want).abs().max()) <= ATOL["bfloat16"]


@pytest.mark.parametrize("case", CASES[:2], ids=lambda c: f"b{c[0]}q{c[1]}kv{c[2]}d{c[3]}p{c[6]}")
def test_early_start_rope_in_decode(case):
    batch, hq, hkv, d, bs, ctxs, pps = case
    q, kn, vn, kc, vc, bt, ctx = _case(4, batch, hq, hkv, d, bs, ctxs)
    g = torch.Generator().manual_seed(2)
    ang = torch.rand(batch, d // 2, generator=g) * 40
    cos = torch.cat([ang.cos(), ang.cos()], 1).to(torch.bfloat16).to(DEV)
    sin = torch.cat([ang.sin(), ang.sin()], 1).to(torch.bfloat16).to(DEV)
    kc1, vc1 = kc.clone(), vc.clone()
    plain = torch.empty(LAYERS, batch, hq, d, device=DEV)
    early = torch.empty_like(plain)
    _step(q, kn, vn, kc, vc, bt, ctx, pps, False, plain, rope=(cos, sin))
    _step(q, kn, vn, kc1, vc1, bt, ctx, pps, True, early, rope=(cos, sin))
    torch.cuda.synchronize()
    assert torch.equal(plain, early)
    assert _sha(kc, vc) == _sha(kc1, vc1)


def test_early_start_in_a_cuda_graph():
    """Three steps captured as one graph (as the benchmark runs them) against the
    same steps launched eagerly without early start."""
    batch, hq, hkv, d, bs, ctxs, pps = CASES[1]
    q, kn, vn, kc, vc, bt, ctx = _case(5, batch, hq, hkv, d, bs, ctxs)
    kc1, vc1 = kc.clone(), vc.clone()
    plain = torch.empty(LAYERS, batch, hq, d, device=DEV)
    graphed = torch.empty_like(plain)
    for _ in range(3):
        _step(q, kn, vn, kc, vc, bt, ctx, pps, False, plain)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _step(q, kn, vn, kc1.clone(), vc1.clone(), bt, ctx, pps, True, graphed)  # warm-up on copies
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(3):
            _step(q, kn, vn, kc1, vc1, bt, ctx, pps, True, graphed)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(plain, graphed)
    assert _sha(kc, vc) == _sha(kc1, vc1)
