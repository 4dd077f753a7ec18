"""Kernel-level parity at the BASELINE configurations' own sizes.

One decode step of one layer of configs 3, 4 and 5, through
the public fused op ``paged_attention_decode(..., k_new=, v_new=)`` (C ABI
pkv_append_decode_run) with the library's default split length, against the
CPU oracle: the append restated from the reference's _paged_kv_update_kernel
(src/triton_kernels/paged_kv.py:253-319) and the 3-pass decode of
_paged_attention_decode_kernel (paged_kv.py:63-251).

  config 3: 16 prompts x group 8 = 128 sequences; each group's 512-token prompt
            lives in 32 pages shared by its 8 block tables (the refcounted
            prompt pages of GRPO groups) followed by U{1..512} private tokens;
  config 4: 1024 sequences, ctx U[1024, 8192], random page permutation;
  config 5: Qwen2.5-7B heads (28 q / 4 kv), 64 sequences, ctx log-U[4096,
            32768]; the default split length is shorter than the longest
            sequences, so the split-K partials and the merge kernel run.

Bars: cache bytes after the append bit-exact, decode
output within max-abs 2e-2 (bf16, fp32 accumulate).
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import ATOL
from grpo_training_engine_b200 import decode_kernel_kind, paged_attention_decode, plan_decode
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
BS, D = 16, 128


def _pool(seed: int, tables: list[list[int]], num_blocks: int, lens, hq: int, hkv: int):
    """Device tensors of one layer: block tables (ids permuted by seed), caches,
    q and the new K / V rows, all N(0,1) bf16."""
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(num_blocks, generator=g)
    B = len(tables)
    max_blocks = max(len(t) for t in tables)
    bt = torch.zeros(B, max_blocks, dtype=torch.int32)
    for i, t in enumerate(tables):
        bt[i, : len(t)] = perm[torch.tensor(t, dtype=torch.long)].int()
    gd = torch.Generator(device=DEV).manual_seed(seed)
    kc = torch.randn(num_blocks, hkv, BS, D, device=DEV, generator=gd).to(torch.bfloat16)
    vc = torch.randn(num_blocks, hkv, BS, D, device=DEV, generator=gd).to(torch.bfloat16)
    q = torch.randn(B, hq, D, device=DEV, generator=gd).to(torch.bfloat16)
    kn = torch.randn(B, hkv, D, device=DEV, generator=gd).to(torch.bfloat16)
    vn = torch.randn(B, hkv, D, device=DEV, generator=gd).to(torch.bfloat16)
    ctx = torch.tensor([int(x) for x in lens], dtype=torch.int32)
    return q, kc, vc, bt.to(DEV), ctx.to(DEV), kn, vn


def _private_tables(lens) -> tuple[list[list[int]], int]:
    tables, nxt = [], 0
    for n in lens:
        p = math.ceil(int(n) / BS)
        tables.append(list(range(nxt, nxt + p)))
        nxt += p
    return tables, nxt


def _step_vs_oracle(q, kc, vc, bt, ctx, kn, vn, expect_merge: bool | None = None):
    """One fused append + decode step on the GPU and by the oracle on copies of
    the same inputs; returns the max-abs decode error and the plan."""
    assert decode_kernel_kind(q, kc) == "tensor_core"
    kc_h, vc_h = kc.cpu(), vc.cpu()
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    plan = plan_decode(ctx, q.shape[1], kc.shape[1], D, BS, bt.shape[1], status=status)
    if expect_merge is not None:
        assert (bt.shape[1] > plan.chosen_pages_per_split()) == expect_merge
    out = paged_attention_decode(q, kc, vc, bt, ctx, plan=plan, k_new=kn, v_new=vn, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    bt_h, ctx_h = bt.cpu(), ctx.cpu()
    oracle.append(kn.cpu(), vn.cpu(), kc_h, vc_h, bt_h, ctx_h - 1)
    assert torch.equal(kc.cpu(), kc_h) and torch.equal(vc.cpu(), vc_h), "appended cache bytes differ"
    ref = oracle.decode(q.cpu(), kc_h, vc_h, bt_h, ctx_h)
    err = float((out.cpu() - ref).abs().max())
    return err, plan


def test_config3_grpo_groups_with_shared_prompt_pages_at_size():
    rs = np.random.RandomState(31)
    groups, group, prompt_pages = 16, 8, 512 // BS
    lens = 512 + rs.randint(1, 513, size=groups * group)  # post-append lengths
    tables, nxt = [], 0
    for gi in range(groups):
        shared = list(range(nxt, nxt + prompt_pages))
        nxt += prompt_pages
        for j in range(group):
            own = math.ceil(int(lens[gi * group + j]) / BS) - prompt_pages
            tables.append(shared + list(range(nxt, nxt + own)))
            nxt += own
    args = _pool(3, tables, nxt, lens, 12, 2)
    bt = args[3].cpu()
    # the 8 rows of a group really share their prompt pages
    assert all(torch.equal(bt[g * group, :prompt_pages], bt[g * group + j, :prompt_pages])
               for g in range(groups) for j in range(group))
    err, _ = _step_vs_oracle(*args)
    assert err <= ATOL["bfloat16"], err


def test_config4_full_batch_one_layer_at_size():
    lens = np.random.RandomState(41).randint(1024, 8193, size=1024)
    tables, nb = _private_tables(lens)
    err, _ = _step_vs_oracle(*_pool(4, tables, nb, lens, 12, 2), expect_merge=False)
    assert err <= ATOL["bfloat16"], err


def test_config5_qwen7b_long_context_split_k_at_size():
    rs = np.random.RandomState(51)
    lens = np.exp(rs.uniform(np.log(4096), np.log(32768), size=64)).astype(np.int64)
    tables, nb = _private_tables(lens)
    err, plan = _step_vs_oracle(*_pool(5, tables, nb, lens, 28, 4), expect_merge=True)
    assert err <= ATOL["bfloat16"], (err, plan.chosen_pages_per_split())


def _expected_split(lens, upi: int, max_blocks: int, sms: int) -> int:
    """The plan kernel's choice of split length (choose_split in pkv_decode.cu),
    restated: for P = lo, lo + 8, ..., top, simulate the snake schedule of the
    units (full splits, then partial splits longest first, upi units per item)
    on the launch's CTAs and take the P whose busiest CTA (pages + 16 per unit,
    + 12 per unit of a split sequence; a partial split's cost at the upper edge
    of its 8-page bin) finishes first, + 16 when a sequence is split; ties to the
    longer split."""
    B = len(lens)
    u0 = B * upi
    hi = min(512, -(-max_blocks // 8) * 8)
    lo = -(-max_blocks * u0 // (16 * sms))
    lo = max(8, -(-lo // 8) * 8, hi - 8 * 63)
    slots = min(sms, B * -(-max_blocks // lo) * upi)
    pages = [math.ceil(int(n) / BS) for n in lens]
    best, best_p = None, hi
    for P in range(lo, hi + 1, 8):
        full = sum(p // P for p in pages)
        # a unit of a split sequence costs 12 pages more (the last partial of a
        # split sequence, and every full split); partial costs are taken at the
        # upper edge of their 8-page bin
        parts = sorted(((p - (p // P) * P + (12 if p // P else 0)) // 8 * 8 + 7
                        for p in pages if max(1, -(-p // P)) > p // P), reverse=True)
        lengths = [P + 12] * full + parts
        units = upi * len(lengths)
        load = [0] * slots
        for r in range(-(-units // slots)):
            for c in range(slots):
                w = r * slots + (slots - 1 - c if r & 1 else c)
                if w < units:
                    load[c] += lengths[w // upi] + 16
        cost = max(load) + (16 if max(pages) > P else 0)
        if best is None or cost < best or (cost == best and P > best_p):
            best, best_p = cost, P
    return best_p


def test_config5_eight_gpu_shard_split_chosen_from_the_lengths():
    """Config 5 strong-scaled to 8 GPUs leaves a GPU 8 long sequences (32 units of
    (sequence, kv head) for 148 SMs): the plan kernel picks the split length
    from their actual lengths by simulating its schedule (not the host's
    all-sequences-at-max-length estimate), and the result still matches the
    oracle."""
    from grpo_training_engine_b200 import _lib
    from grpo_training_engine_b200.sharding import lpt_assign

    rs = np.random.RandomState(51)
    lens_all = np.exp(rs.uniform(np.log(4096), np.log(32768), size=64)).astype(np.int64)
    lens = [int(lens_all[i]) for i in lpt_assign(lens_all.tolist(), 8)[0]]
    tables, nb = _private_tables(lens)
    args = _pool(6, tables, nb, lens, 28, 4)
    max_blocks = args[3].shape[1]
    err, plan = _step_vs_oracle(*args)
    assert err <= ATOL["bfloat16"], err
    host = _lib.load().pkv_decode_pages_per_split(len(lens), 28, 4, D, max_blocks, 0)
    chosen = plan.chosen_pages_per_split()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert chosen == _expected_split(lens, 4, max_blocks, sms), (chosen, host)
    assert chosen != host
