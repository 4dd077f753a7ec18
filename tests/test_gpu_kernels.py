"""Parity of the CUDA kernels (through the C ABI) with the reference and the oracle.

Bars: append, prompt append and gather bit-exact;
decode output within max-abs 1e-5 of the reference arithmetic for fp32
caches and 2e-2 for bf16/fp16 caches (fp32 accumulation).
"""

from __future__ import annotations

import hashlib
import math

import numpy as np
import pytest
import torch

import cases
from conftest import ATOL, load_golden
from grpo_training_engine_b200 import (
    decode_kernel_kind,
    gather_kv,
    paged_attention_decode,
    paged_kv_append,
    paged_kv_append_prompt,
    plan_decode,
)
from grpo_training_engine_b200 import _lib
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"
RAW = {torch.float32: torch.int32, torch.bfloat16: torch.int16, torch.float16: torch.int16}


def _sha(*tensors: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(np.ascontiguousarray(t.detach().cpu().contiguous().view(RAW[t.dtype]).numpy()).tobytes())
    return h.hexdigest()


def _maxabs(a: torch.Tensor, b) -> float:
    b = torch.as_tensor(b)
    return float((a.detach().cpu().float() - b.float()).abs().max()) if a.numel() else 0.0


# ------------------------------------------------------------------ golden vectors
@pytest.mark.parametrize("name", [c["name"] for c in cases.CASES])
@pytest.mark.parametrize("mode", ["fast", "exact", "generic"])
def test_golden_append_and_decode(name, mode):
    case = cases.BY_NAME[name]
    ref_out, meta = load_golden(name)
    t = cases.to_torch(cases.make_inputs(case), case["dtype"], device=DEV)
    ctx = t["context_lens"]
    if case["append"]:
        paged_kv_append(t["k_new"], t["v_new"], t["k_cache"], t["v_cache"], t["block_tables"], ctx)
        ctx = ctx + 1
    assert _sha(t["k_cache"], t["v_cache"]) == meta["cache_after_append_sha"]
    out = paged_attention_decode(t["q"], t["k_cache"], t["v_cache"], t["block_tables"], ctx,
                                 force_generic=mode == "generic", exact=mode == "exact")
    torch.cuda.synchronize()
    assert _maxabs(out, ref_out) <= ATOL[case["dtype"]], _maxabs(out, ref_out)
    if mode != "fast" or case["dtype"] == "float32":
        # exact-P tensor-core kernel and the CUDA-core kernel track fp32 closely
        assert _maxabs(out, ref_out) <= 2e-4, _maxabs(out, ref_out)


@pytest.mark.parametrize("name", [c["name"] for c in cases.CASES if c.get("prompt_steps")])
def test_golden_prompt_scatter(name):
    case = cases.BY_NAME[name]
    _, meta = load_golden(name)
    t = cases.to_torch(cases.make_inputs(case), case["dtype"], device=DEV)
    kc = torch.zeros_like(t["k_cache"])
    vc = torch.zeros_like(t["v_cache"])
    paged_kv_append_prompt(t["prompt_k"], t["prompt_v"], kc, vc, t["block_tables"])
    assert _sha(kc, vc) == meta["prompt_cache_sha"]


def test_bf16_golden_selects_tensor_core_kernel():
    case = cases.BY_NAME["bf16_qwen7b_g7"]
    t = cases.to_torch(cases.make_inputs(case), case["dtype"], device=DEV)
    assert decode_kernel_kind(t["q"], t["k_cache"]) == "tensor_core"
    assert decode_kernel_kind(t["q"], t["k_cache"], force_generic=True) == "cuda_core"


# ------------------------------------------------------------- random vs oracle
def _random_case(seed, batch, hq, hkv, d, bs, ctxs, dtype, num_blocks=None, spare=3):
    g = torch.Generator().manual_seed(seed)
    max_blocks = max(1, max(math.ceil(c / bs) for c in ctxs) + 1)
    num_blocks = num_blocks or batch * max_blocks + spare
    perm = torch.randperm(num_blocks, generator=g)[: batch * max_blocks].reshape(batch, max_blocks).int()
    q = torch.randn(batch, hq, d, generator=g).to(dtype)
    kc = torch.randn(num_blocks, hkv, bs, d, generator=g).to(dtype)
    vc = torch.randn(num_blocks, hkv, bs, d, generator=g).to(dtype)
    ctx = torch.tensor(ctxs, dtype=torch.int32)
    return q, kc, vc, perm, ctx


DECODE_SHAPES = [
    # (batch, hq, hkv, head_dim, block_size, dtype, ctxs)
    (4, 12, 2, 128, 16, torch.bfloat16, [1, 16, 17, 777]),          # 1.5B geometry
    (3, 28, 4, 128, 16, torch.bfloat16, [5000, 33, 2048]),           # 7B geometry
    (2, 8, 8, 128, 16, torch.bfloat16, [100, 300]),                  # replicated heads (G=1)
    (2, 32, 2, 128, 16, torch.bfloat16, [129, 64]),                  # G=16 (one full MMA tile)
    (2, 40, 2, 64, 16, torch.float16, [500, 1]),                     # G=20 -> two head groups
    (2, 16, 2, 64, 16, torch.bfloat16, [0, 95]),                     # empty context
    (3, 12, 2, 128, 16, torch.float32, [37, 128, 300]),              # fp32 -> CUDA cores
    (2, 6, 3, 96, 8, torch.bfloat16, [50, 9]),                       # odd head_dim / block size
    (2, 4, 1, 256, 32, torch.float16, [200, 31]),                    # wide heads
    (2, 2, 2, 8, 4, torch.float32, [6, 3]),                          # reference test geometry
]


@pytest.mark.parametrize("shape", DECODE_SHAPES, ids=lambda s: f"b{s[0]}q{s[1]}kv{s[2]}d{s[3]}bs{s[4]}")
@pytest.mark.parametrize("splits", [0, 1, 5])
def test_decode_matches_oracle(shape, splits):
    batch, hq, hkv, d, bs, dtype, ctxs = shape
    q, kc, vc, bt, ctx = _random_case(11, batch, hq, hkv, d, bs, ctxs, dtype)
    ref = oracle.decode(q, kc, vc, bt, ctx)
    tol = ATOL[str(dtype).split(".")[1]]
    for force_generic in (False, True):
        out = paged_attention_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), ctx.to(DEV),
                                     num_splits=splits, force_generic=force_generic)
        assert _maxabs(out, ref) <= tol, (force_generic, _maxabs(out, ref))


def test_exact_mode_precision_and_fast_mode_error_size():
    q, kc, vc, bt, ctx = _random_case(13, 8, 12, 2, 128, 16, [4000, 17, 900, 1, 2048, 300, 5000, 64],
                                      torch.bfloat16)
    ref = oracle.decode(q, kc, vc, bt, ctx)
    args = [x.to(DEV) for x in (q, kc, vc, bt, ctx)]
    exact = paged_attention_decode(*args, exact=True)
    fast = paged_attention_decode(*args)
    assert _maxabs(exact, ref) <= 2e-4
    assert _maxabs(fast, ref) <= 2e-2
    assert decode_kernel_kind(args[0], args[1]) == "tensor_core"


@pytest.mark.parametrize("pages_per_split", [1, 2, 8, 64])
def test_split_invariance_and_determinism(pages_per_split):
    q, kc, vc, bt, ctx = _random_case(5, 6, 12, 2, 128, 16, [3000, 1, 17, 512, 4096, 2049], torch.bfloat16)
    args = [x.to(DEV) for x in (q, kc, vc, bt, ctx)]
    a = paged_attention_decode(*args, pages_per_split=pages_per_split)
    b = paged_attention_decode(*args, pages_per_split=pages_per_split)
    assert torch.equal(a, b)  # no atomics in the arithmetic: bitwise reproducible
    whole = paged_attention_decode(*args, pages_per_split=4096)
    assert _maxabs(a, whole.cpu()) < 2e-3
    ref = oracle.decode(q, kc, vc, bt, ctx)
    assert _maxabs(a, ref) <= 2e-2


def test_strided_views_and_pool_layers():
    """Caches as layers of a 5-D pool, q as a slice, out as a strided view."""
    L, nb, hkv, bs, d, hq, batch = 3, 40, 2, 16, 128, 12, 3
    g = torch.Generator().manual_seed(2)
    pool = torch.randn(2, L, nb, hkv, bs, d, generator=g).to(torch.bfloat16)
    big_q = torch.randn(batch, hq * 2, d, generator=g).to(torch.bfloat16)
    bt = torch.randperm(nb, generator=g)[: batch * 10].reshape(batch, 10).int()
    ctx = torch.tensor([150, 7, 160], dtype=torch.int32)
    pool_d = pool.to(DEV)
    out_big = torch.zeros(batch, hq, d * 2, device=DEV)
    for layer in range(L):
        kc, vc = pool_d[0, layer], pool_d[1, layer]
        q = big_q[:, ::2].to(DEV)  # non-contiguous heads
        out = out_big[:, :, ::2]
        paged_attention_decode(q, kc, vc, bt.to(DEV), ctx.to(DEV), out=out)
        ref = oracle.decode(big_q[:, ::2], pool[0, layer], pool[1, layer], bt, ctx)
        assert _maxabs(out, ref) <= 2e-2
        assert not out_big[:, :, 1::2].any()


def test_plan_reuse_across_layers():
    q, kc, vc, bt, ctx = _random_case(8, 5, 12, 2, 128, 16, [900, 3, 64, 65, 1500], torch.bfloat16)
    qd, kd, vd, btd, cd = (x.to(DEV) for x in (q, kc, vc, bt, ctx))
    plan = plan_decode(cd, 12, 2, 128, 16, bt.shape[1], pages_per_split=8)
    for _ in range(3):
        out = paged_attention_decode(qd, kd, vd, btd, cd, plan=plan)
        assert _maxabs(out, oracle.decode(q, kc, vc, bt, ctx)) <= 2e-2


def test_full_scale_properties():
    """Size-independent properties at config-4 lengths: constant V gives V; zero K gives mean(V)."""
    batch, hq, hkv, d, bs = 32, 12, 2, 128, 16
    g = torch.Generator().manual_seed(9)
    ctxs = torch.randint(1024, 8193, (batch,), generator=g)
    max_blocks = int(math.ceil(ctxs.max().item() / bs))
    nb = batch * max_blocks
    bt = torch.randperm(nb, generator=g).reshape(batch, max_blocks).int().to(DEV)
    q = torch.randn(batch, hq, d, generator=g).to(torch.bfloat16).to(DEV)
    kc = torch.randn(nb, hkv, bs, d, generator=g).to(torch.bfloat16).to(DEV)
    vc = torch.full((nb, hkv, bs, d), 0.75, dtype=torch.bfloat16, device=DEV)
    ctx = ctxs.int().to(DEV)
    out = paged_attention_decode(q, kc, vc, bt, ctx)
    assert float((out - 0.75).abs().max()) < 4e-3
    kz = torch.zeros_like(kc)
    vr = torch.randn(nb, hkv, bs, d, generator=g).to(torch.bfloat16).to(DEV)
    out = paged_attention_decode(q, kz, vr, bt, ctx)
    dense_v, _ = gather_kv(vr, vr, bt, ctx)
    mean = dense_v.float().sum(dim=2) / ctx.view(-1, 1, 1).float()
    exp = mean.repeat_interleave(hq // hkv, dim=1)
    assert float((out - exp).abs().max()) < 1e-3


def test_large_ragged_batch_vs_oracle():
    q, kc, vc, bt, ctx = _random_case(21, 48, 12, 2, 128, 16,
                                      torch.randint(1024, 8193, (48,), generator=torch.Generator().manual_seed(1)).tolist(),
                                      torch.bfloat16)
    out = paged_attention_decode(*(x.to(DEV) for x in (q, kc, vc, bt, ctx)))
    assert _maxabs(out, oracle.decode(q, kc, vc, bt, ctx)) <= 2e-2


def test_out_of_range_inputs_are_flagged_not_faulted():
    q, kc, vc, bt, ctx = _random_case(3, 3, 12, 2, 128, 16, [40, 40, 40], torch.bfloat16)
    bad_bt = bt.clone()
    bad_bt[1, 1] = kc.shape[0] + 5  # page id past the pool
    bad_bt[2, 0] = -1
    for force_generic in (False, True):
        status = torch.zeros(1, dtype=torch.int32, device=DEV)
        out = paged_attention_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bad_bt.to(DEV), ctx.to(DEV),
                                     status=status, force_generic=force_generic)
        assert int(status.item()) & _lib.DEV_PAGE_OUT_OF_RANGE
        # invalid pages are skipped, exactly like the oracle does
        assert _maxabs(out, oracle.decode(q, kc, vc, bad_bt, ctx)) <= 2e-2
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    too_long = torch.tensor([40, 10_000, -3], dtype=torch.int32)
    out = paged_attention_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), too_long.to(DEV), status=status)
    assert int(status.item()) & _lib.DEV_CTX_OUT_OF_RANGE
    assert _maxabs(out, oracle.decode(q, kc, vc, bt, too_long)) <= 2e-2
    # append past the table is skipped and flagged
    status.zero_()
    kn = torch.randn(3, 2, 128, dtype=torch.bfloat16, device=DEV)
    before = kc.to(DEV)
    after = before.clone()
    paged_kv_append(kn, kn.clone(), after, after.clone(), bt.to(DEV), torch.tensor([10_000, -1, 10_000], dtype=torch.int32, device=DEV), status=status)
    assert int(status.item()) & _lib.DEV_CTX_OUT_OF_RANGE
    assert torch.equal(before, after)


# ------------------------------------------------------- fused append + decode
FUSED_SHAPES = [
    # (batch, hq, hkv, head_dim, block_size, dtype, post-append ctxs)
    (4, 12, 2, 128, 16, torch.bfloat16, [1, 16, 17, 777]),    # token opens / fills / first page
    (3, 28, 4, 128, 16, torch.bfloat16, [5000, 33, 2048]),     # 7B geometry, long splits
    (2, 40, 2, 64, 16, torch.float16, [500, 1]),               # two head groups read the page
    (2, 16, 2, 64, 16, torch.bfloat16, [0, 95]),               # an empty sequence appends nothing
    (3, 12, 2, 128, 16, torch.float32, [37, 128, 300]),        # fp32: append kernel + CUDA cores
    (2, 6, 3, 96, 8, torch.bfloat16, [50, 9]),                 # CUDA-core kernel shape
]


def _separate_append_then_decode(q, kn, vn, kc, vc, bt, ctx, **kw):
    """The reference's per-layer pair: append at the pre-append length, decode over ctx."""
    live = (ctx > 0).nonzero().flatten()
    if live.numel():
        paged_kv_append(kn[live], vn[live], kc, vc, bt[live], (ctx - 1)[live])
    return paged_attention_decode(q, kc, vc, bt, ctx, **kw)


@pytest.mark.parametrize("shape", FUSED_SHAPES, ids=lambda s: f"b{s[0]}q{s[1]}kv{s[2]}d{s[3]}bs{s[4]}")
@pytest.mark.parametrize("splits", [0, 3])
def test_fused_append_decode_equals_separate_calls(shape, splits):
    batch, hq, hkv, d, bs, dtype, ctxs = shape
    q, kc, vc, bt, ctx = _random_case(21, batch, hq, hkv, d, bs, ctxs, dtype)
    g = torch.Generator().manual_seed(5)
    kn = torch.randn(batch, hkv, d, generator=g).to(dtype)
    vn = torch.randn(batch, hkv, d, generator=g).to(dtype)
    q, kn, vn, bt, ctx = (t.to(DEV) for t in (q, kn, vn, bt, ctx))
    kc1, vc1 = kc.to(DEV), vc.to(DEV)
    kc2, vc2 = kc1.clone(), vc1.clone()
    out1 = _separate_append_then_decode(q, kn, vn, kc1, vc1, bt, ctx, num_splits=splits)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out2 = paged_attention_decode(q, kc2, vc2, bt, ctx, num_splits=splits, k_new=kn, v_new=vn, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert _sha(kc1, vc1) == _sha(kc2, vc2)  # the same cache bytes
    assert torch.equal(out1, out2)           # the same tiles in smem, the same arithmetic
    ref = oracle.decode(q.cpu(), kc1.cpu(), vc1.cpu(), bt.cpu(), ctx.cpu())
    assert _maxabs(out2, ref) <= ATOL[str(dtype).split(".")[1]]


def test_fused_append_decode_with_strided_new_rows_and_plan_reuse():
    # new rows with a padded head stride (head_dim contiguous) take the one-launch
    # route, head_dim-strided rows the append-kernel route; one plan, 3 layers
    batch, hq, hkv, d = 5, 12, 2, 128
    ctxs = [300, 1, 64, 65, 1000]
    q, kc, vc, bt, ctx = _random_case(8, batch, hq, hkv, d, 16, ctxs, torch.bfloat16)
    pool_k = torch.stack([kc, kc.roll(1, 0), kc.roll(2, 0)]).to(DEV)
    pool_v = torch.stack([vc, vc.roll(3, 0), vc.roll(1, 0)]).to(DEV)
    g = torch.Generator().manual_seed(9)
    padded = torch.randn(3, batch, hkv, 2 * d, generator=g).to(torch.bfloat16).to(DEV)[..., :d]
    strided = torch.randn(3, batch, d, hkv, generator=g).to(torch.bfloat16).to(DEV).transpose(2, 3)
    q, bt, ctx = q.to(DEV), bt.to(DEV), ctx.to(DEV)
    plan = plan_decode(ctx, hq, hkv, d, 16, bt.shape[1], pages_per_split=8)
    for layer in range(3):
        for new in (padded[layer], strided[layer]):
            pk, pv = pool_k[layer].clone(), pool_v[layer].clone()
            out = paged_attention_decode(q, pk, pv, bt, ctx, plan=plan, k_new=new, v_new=new)
            rk, rv = pool_k[layer].clone(), pool_v[layer].clone()
            ref = _separate_append_then_decode(q, new.contiguous(), new.contiguous(), rk, rv, bt, ctx,
                                               pages_per_split=8)
            assert _sha(pk, pv) == _sha(rk, rv)
            assert torch.equal(out, ref)


def test_fused_append_out_of_range_page_is_flagged_and_skipped():
    q, kc, vc, bt, ctx = _random_case(3, 3, 12, 2, 128, 16, [40, 17, 5], torch.bfloat16)
    bad = bt.clone()
    bad[0, 2] = 10_000  # page of sequence 0's new token (position 39)
    kn = torch.randn(3, 2, 128).to(torch.bfloat16)
    kd, vd = kc.to(DEV), vc.to(DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = paged_attention_decode(q.to(DEV), kd, vd, bad.to(DEV), ctx.to(DEV), k_new=kn.to(DEV),
                                 v_new=kn.to(DEV), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & _lib.DEV_PAGE_OUT_OF_RANGE
    # sequences 1 and 2 got their tokens; sequence 0's bad page is skipped in both cache and decode
    kc2, vc2 = kc.clone(), vc.clone()
    oracle.append(kn[1:], kn[1:], kc2, vc2, bad[1:], ctx[1:] - 1)
    assert _sha(kd, vd) == _sha(kc2, vc2)
    assert _maxabs(out, oracle.decode(q, kc2, vc2, bad, ctx)) <= 2e-2


# ---------------------------------------------------------------- append / gather
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("d", [8, 6, 128])
def test_append_gather_bit_exact(dtype, d):
    g = torch.Generator().manual_seed(4)
    batch, heads, bs, nb, mb = 5, 3, 8, 40, 6
    bt = torch.randperm(nb, generator=g)[: batch * mb].reshape(batch, mb).int()
    ctx = torch.tensor([0, 7, 8, 30, 47], dtype=torch.int32)
    kc = torch.randn(nb, heads, bs, d, generator=g).to(dtype)
    vc = torch.randn(nb, heads, bs, d, generator=g).to(dtype)
    kn = torch.randn(batch, heads, d, generator=g).to(dtype)
    vn = torch.randn(batch, heads, d, generator=g).to(dtype)
    kd, vd = kc.to(DEV), vc.to(DEV)
    paged_kv_append(kn.to(DEV), vn.to(DEV), kd, vd, bt.to(DEV), ctx.to(DEV))
    oracle.append(kn, vn, kc, vc, bt, ctx)
    assert _sha(kd, vd) == _sha(kc, vc)
    k1, v1 = gather_kv(kd, vd, bt.to(DEV), (ctx + 1).to(DEV))
    k2, v2 = oracle.gather(kc, vc, bt, ctx + 1)
    assert _sha(k1, v1) == _sha(k2, v2)


def test_append_prompt_with_offsets_and_lengths():
    g = torch.Generator().manual_seed(6)
    batch, heads, bs, nb, mb, d, T = 3, 2, 16, 30, 8, 128, 50
    bt = torch.randperm(nb, generator=g)[: batch * mb].reshape(batch, mb).int()
    k = torch.randn(batch, heads, T, d, generator=g).to(torch.bfloat16)
    v = torch.randn(batch, heads, T, d, generator=g).to(torch.bfloat16)
    start = torch.tensor([0, 5, 70], dtype=torch.int32)
    lens = torch.tensor([50, 13, 40], dtype=torch.int32)
    kc = torch.zeros(nb, heads, bs, d, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    kd, vd = kc.to(DEV), vc.to(DEV)
    paged_kv_append_prompt(k.to(DEV), v.to(DEV), kd, vd, bt.to(DEV), start.to(DEV), lens.to(DEV))
    oracle.append_prompt(k, v, kc, vc, bt, start, lens)
    assert _sha(kd, vd) == _sha(kc, vc)


def test_config2_append_gather_round_trip():
    """28 layers x 2 kv heads x 128, bs 16, 8 sequences; 512-token
    prompt written in bulk, then 512 single-token appends; gather must return
    every written token bit for bit."""
    L, batch, hkv, d, bs, P, N = 28, 8, 2, 128, 16, 512, 512
    pages = (P + N) // bs
    g = torch.Generator(device=DEV).manual_seed(22)
    nb = batch * pages + 7
    perm = torch.randperm(nb, device=DEV, generator=g)[: batch * pages].reshape(batch, pages).int()
    k_pool = torch.zeros(L, nb, hkv, bs, d, dtype=torch.bfloat16, device=DEV)
    v_pool = torch.zeros_like(k_pool)
    prompt_k = torch.randn(L, batch, hkv, P, d, device=DEV, generator=g).to(torch.bfloat16)
    prompt_v = torch.randn(L, batch, hkv, P, d, device=DEV, generator=g).to(torch.bfloat16)
    new_k = torch.randn(N, L, batch, hkv, d, device=DEV, generator=g).to(torch.bfloat16)
    new_v = torch.randn(N, L, batch, hkv, d, device=DEV, generator=g).to(torch.bfloat16)
    for layer in range(L):
        paged_kv_append_prompt(prompt_k[layer], prompt_v[layer], k_pool[layer], v_pool[layer], perm)
    ctx = torch.full((batch,), P, dtype=torch.int32, device=DEV)
    for step in range(N):
        for layer in range(L):
            paged_kv_append(new_k[step, layer], new_v[step, layer], k_pool[layer], v_pool[layer], perm, ctx)
        ctx += 1
    for layer in range(L):
        kg, vg = gather_kv(k_pool[layer], v_pool[layer], perm, ctx)
        exp_k = torch.cat([prompt_k[layer], new_k[:, layer].permute(1, 2, 0, 3)], dim=2)
        exp_v = torch.cat([prompt_v[layer], new_v[:, layer].permute(1, 2, 0, 3)], dim=2)
        assert torch.equal(kg.view(torch.int16), exp_k.view(torch.int16))
        assert torch.equal(vg.view(torch.int16), exp_v.view(torch.int16))
    # and one layer against the oracle's scatter of the same data
    layer = 5
    kc = torch.zeros(nb, hkv, bs, d, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    full_k = torch.cat([prompt_k[layer], new_k[:, layer].permute(1, 2, 0, 3)], dim=2).cpu()
    full_v = torch.cat([prompt_v[layer], new_v[:, layer].permute(1, 2, 0, 3)], dim=2).cpu()
    oracle.append_prompt(full_k, full_v, kc, vc, perm.cpu())
    assert _sha(k_pool[layer], v_pool[layer]) == _sha(kc, vc)


@pytest.mark.parametrize("shape", [s for s in DECODE_SHAPES if s[5] != torch.float32],
                         ids=lambda s: f"b{s[0]}q{s[1]}kv{s[2]}d{s[3]}bs{s[4]}")
@pytest.mark.parametrize("splits", [0, 3])
def test_out_in_q_dtype_equals_cast_of_fp32_out(shape, splits):
    """out_dtype=q.dtype writes what .to(q.dtype) of the fp32 output holds, on every
    kernel (tensor-core, CUDA-core, split-K merge) and with the fused append."""
    batch, hq, hkv, d, bs, dtype, ctxs = shape
    q, kc, vc, bt, ctx = (t.to(DEV) for t in _random_case(31, batch, hq, hkv, d, bs, ctxs, dtype))
    for force_generic in (False, True):
        ref = paged_attention_decode(q, kc, vc, bt, ctx, num_splits=splits, force_generic=force_generic)
        got = paged_attention_decode(q, kc, vc, bt, ctx, num_splits=splits, force_generic=force_generic,
                                     out_dtype=dtype)
        assert got.dtype == dtype and torch.equal(got, ref.to(dtype)), force_generic
    # strided 16-bit out (no vector stores) and the fused append
    g = torch.Generator().manual_seed(6)
    kn, vn = (torch.randn(batch, hkv, d, generator=g).to(dtype).to(DEV) for _ in range(2))
    kc2, vc2 = kc.clone(), vc.clone()
    ref = paged_attention_decode(q, kc, vc, bt, ctx, num_splits=splits, k_new=kn, v_new=vn)
    wide = torch.zeros(batch, hq, d + 4, dtype=dtype, device=DEV)  # rows 4-byte but not 8-byte aligned
    got = paged_attention_decode(q, kc2, vc2, bt, ctx, num_splits=splits, k_new=kn, v_new=vn,
                                 out=wide[:, :, 2:d + 2], out_dtype=dtype)
    assert torch.equal(got, ref.to(dtype)) and not wide[:, :, :2].any() and not wide[:, :, d + 2:].any()
    with pytest.raises(ValueError, match="out_dtype"):
        paged_attention_decode(q, kc, vc, bt, ctx, out_dtype=torch.float64)


ROPE_SHAPES = [
    (4, 12, 2, 128, 16, torch.bfloat16, [1, 16, 17, 777]),    # 1.5B geometry
    (3, 28, 4, 128, 16, torch.bfloat16, [5000, 33, 2048]),     # 7B geometry (split-K)
    (2, 40, 2, 64, 16, torch.float16, [500, 1]),               # two head groups
    (2, 16, 2, 64, 16, torch.bfloat16, [0, 95]),               # empty context
]


@pytest.mark.parametrize("shape", ROPE_SHAPES, ids=lambda s: f"b{s[0]}q{s[1]}kv{s[2]}d{s[3]}")
@pytest.mark.parametrize("splits", [0, 3])
def test_rope_in_decode_equals_rope_then_fused_decode(shape, splits):
    """RoPE inside the decode launch against rope_qk followed by the fused append +
    decode, also when q / k / v are column views of one stacked projection
    output: the rotated K row lands in the cache bit for bit, and both outputs
    match the oracle on the rotated inputs. For head_dim 64 both calls run the
    same kernel configuration and agree bit for bit; for head_dim 128 the RoPE
    launch runs 7 consumer warps (its registers allow no more) and the plain one
    9, so pages meet the softmax in other warps and the bf16-rounded weights
    differ within the decode tolerance."""
    from grpo_training_engine_b200 import ops

    batch, hq, hkv, d, bs, dtype, ctxs = shape
    q, kc, vc, bt, ctx = _random_case(41, batch, hq, hkv, d, bs, ctxs, dtype)
    g = torch.Generator().manual_seed(7)
    qkv = (torch.randn(batch, (hq + 2 * hkv) * d, generator=g) * 2).to(dtype).to(DEV)
    ang = torch.rand(batch, d // 2, generator=g) * 50
    cos = torch.cat([ang.cos(), ang.cos()], 1).to(dtype).to(DEV)
    sin = torch.cat([ang.sin(), ang.sin()], 1).to(dtype).to(DEV)
    bt, ctx = bt.to(DEV), ctx.to(DEV)
    q_lin, k_lin, v_lin = qkv[:, :hq * d], qkv[:, hq * d:(hq + hkv) * d], qkv[:, (hq + hkv) * d:]
    kc1, vc1 = kc.to(DEV), vc.to(DEV)
    kc2, vc2 = kc1.clone(), vc1.clone()
    q1, k1 = ops.rope_qk(q_lin, k_lin, cos, sin, hq, hkv, d)
    v1 = v_lin.contiguous().view(batch, hkv, d)
    ref = paged_attention_decode(q1, kc1, vc1, bt, ctx, num_splits=splits, k_new=k1, v_new=v1)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    got = paged_attention_decode(q_lin.view(batch, hq, d), kc2, vc2, bt, ctx, num_splits=splits,
                                 k_new=k_lin.view(batch, hkv, d), v_new=v_lin.view(batch, hkv, d),
                                 rope=(cos, sin), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert _sha(kc1, vc1) == _sha(kc2, vc2)
    want = oracle.decode(q1.cpu(), kc1.cpu(), vc1.cpu(), bt.cpu(), ctx.cpu())
    tol = ATOL[str(dtype).split(".")[1]]
    assert _maxabs(got, want) <= tol and _maxabs(ref, want) <= tol, (_maxabs(got, want), _maxabs(ref, want))
    if d == 64:
        assert torch.equal(got, ref)
    # contiguous inputs, 16-bit output: the cast of the fp32 output of the same launch
    got16 = paged_attention_decode(q_lin.contiguous().view(batch, hq, d), kc2.clone(), vc2.clone(), bt, ctx,
                                   num_splits=splits, k_new=k_lin.contiguous().view(batch, hkv, d), v_new=v1,
                                   rope=(cos, sin), out_dtype=dtype)
    assert torch.equal(got16, got.to(dtype))


def test_rope_in_decode_refuses_what_it_cannot_serve():
    from grpo_training_engine_b200 import _lib

    q, kc, vc, bt, ctx = (t.to(DEV) for t in _random_case(3, 2, 4, 2, 8, 4, [5, 9], torch.float32))
    kn = torch.zeros(2, 2, 8, device=DEV)
    cs = torch.ones(2, 8, device=DEV)
    with pytest.raises(_lib.PkvError, match="RoPE in the decode"):  # fp32: CUDA-core kernel
        paged_attention_decode(q, kc, vc, bt, ctx, k_new=kn, v_new=kn.clone(), rope=(cs, cs))
    with pytest.raises(ValueError, match="rope needs k_new"):
        paged_attention_decode(q, kc, vc, bt, ctx, rope=(cs, cs))


@pytest.mark.parametrize(
    "dtype,d,hq,hkv,kw",
    [
        (torch.bfloat16, 128, 12, 2, {}),
        (torch.float16, 64, 12, 2, {}),
        (torch.bfloat16, 128, 16, 1, {}),  # 16 query heads per KV head: two head tiles
        (torch.bfloat16, 128, 12, 2, {"exact": True}),
        (torch.bfloat16, 128, 12, 2, {"force_generic": True}),
        (torch.float32, 128, 12, 2, {}),  # fp32 cache: the generic kernel
    ],
)
def test_nan_in_unused_page_slots_does_not_leak(dtype, d, hq, hkv, kw):
    """Slots past a sequence's context in its last page may hold anything (a cache
    from torch.empty); the reference's masked loads never read them. NaN / Inf there
    must not reach the output: same bits as with zeros there, fused append included,
    in every kernel variant."""
    batch, bs = 3, 16
    ctxs = [5, 40, 17]
    q, kc, vc, bt, ctx = _random_case(51, batch, hq, hkv, d, bs, ctxs, dtype)
    q, kc, vc, bt, ctx = (t.to(DEV) for t in (q, kc, vc, bt, ctx))
    dirty_k, dirty_v = kc.clone(), vc.clone()
    for b, c in enumerate(ctxs):
        page = int(bt[b, c // bs])
        dirty_k[page, :, c % bs:] = float("nan")
        dirty_v[page, :, c % bs:] = float("inf")
        kc[page, :, c % bs:] = 0
        vc[page, :, c % bs:] = 0
    for splits in (0, 2):
        clean = paged_attention_decode(q, kc, vc, bt, ctx, num_splits=splits, **kw)
        got = paged_attention_decode(q, dirty_k, dirty_v, bt, ctx, num_splits=splits, **kw)
        assert torch.isfinite(got).all() and torch.equal(got, clean)
    # fused append: the new token lands at ctx - 1 of the post-append length
    g = torch.Generator().manual_seed(2)
    kn, vn = (torch.randn(batch, hkv, d, generator=g).to(dtype).to(DEV) for _ in range(2))
    post = ctx + 1
    clean = paged_attention_decode(q, kc.clone(), vc.clone(), bt, post, k_new=kn, v_new=vn, **kw)
    got = paged_attention_decode(q, dirty_k.clone(), dirty_v.clone(), bt, post, k_new=kn, v_new=vn, **kw)
    assert torch.isfinite(got).all() and torch.equal(got, clean)
