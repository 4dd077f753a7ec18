"""Host-side logic that needs no GPU: the reference's validation contract,
the façade's routing, sampling helpers, the page pool and the sharder."""

from __future__ import annotations

import math

import pytest
import torch

import grpo_training_engine_b200 as pkg
from grpo_training_engine_b200 import paged_kv
from grpo_training_engine_b200.kv_pool import KVPagePool, PoolExhausted
from grpo_training_engine_b200.sharding import imbalance, lpt_assign, shard_groups


# ----------------------------------------------------------- validation contract
def _args(**over):
    a = dict(
        input_ids=torch.zeros(2, 3, dtype=torch.long),
        k_cache=torch.zeros(4, 2, 4, 8, dtype=torch.bfloat16),
        v_cache=torch.zeros(4, 2, 4, 8, dtype=torch.bfloat16),
        block_tables=torch.zeros(2, 2, dtype=torch.int32),
        context_lens=torch.zeros(2, dtype=torch.int32),
    )
    a.update(over)
    return a


@pytest.mark.parametrize(
    "over, msg",
    [
        (dict(input_ids=torch.zeros(3, dtype=torch.long)), "input_ids must be \\[batch, seq_len\\]"),
        (dict(k_cache=torch.zeros(4, 2, 4)), "k_cache/v_cache must be \\[num_blocks, heads, block, head_dim\\]."),
        (dict(v_cache=torch.zeros(4, 2, 4, 4, dtype=torch.bfloat16)), "identical shapes"),
        (dict(block_tables=torch.zeros(2, dtype=torch.int32)), "block_tables must be \\[batch, max_blocks\\]"),
        (dict(context_lens=torch.zeros(2, 1, dtype=torch.int32)), "context_lens must be \\[batch\\]"),
        (dict(block_tables=torch.zeros(3, 2, dtype=torch.int32)), "block_tables batch dimension"),
        (dict(context_lens=torch.zeros(3, dtype=torch.int32)), "context_lens batch dimension"),
        (dict(), "inputs and caches must be on CUDA device."),
    ],
)
def test_validate_inputs_messages(over, msg):
    with pytest.raises(ValueError, match=msg):
        paged_kv._validate_inputs(**_args(**over))


def test_low_level_rejects_nonpositive_tokens():
    a = _args()
    with pytest.raises(ValueError, match="max_new_tokens must be > 0, got 0."):
        paged_kv.paged_kv_decode(a["input_ids"], a["k_cache"], a["v_cache"], a["block_tables"],
                                 a["context_lens"], lambda x: x, lambda x: x, max_new_tokens=0)


def _fake_low_level(monkeypatch, script, vocab=16):
    """The low-level driver with its kernels replaced by fakes that record the
    lengths they get, and logits_fn replaced by a script of greedy tokens (one
    row of tokens per step). Returns (run, calls)."""
    calls = []

    def fake_decode(q, k_cache, v_cache, block_tables, context_lens, scale=None, k_new=None, v_new=None, **kw):
        calls.append(("fused" if k_new is not None else "decode", context_lens.tolist()))
        return torch.zeros(q.shape, dtype=torch.float32)

    def fake_append(k_new, v_new, k_cache, v_cache, block_tables, context_lens):
        calls.append(("append", context_lens.tolist()))

    monkeypatch.setattr(paged_kv.ops, "paged_attention_decode", fake_decode)
    monkeypatch.setattr(paged_kv.ops, "paged_kv_append", fake_append)
    monkeypatch.setattr(paged_kv, "_validate_inputs", lambda *a: (2, 4, 8, 64))
    step = iter(script)

    def logits_fn(attn):
        return torch.nn.functional.one_hot(torch.tensor(next(step)), vocab).float()

    def run(ctx, eos, new):
        a = _args()
        ids = torch.tensor([[13, 1], [14, 2]])
        q = torch.zeros(2, 2, 8, dtype=torch.bfloat16)
        return paged_kv.paged_kv_decode(ids, a["k_cache"], a["v_cache"], a["block_tables"],
                                        torch.tensor(ctx, dtype=torch.int32), lambda t: (q, q, q), logits_fn,
                                        max_new_tokens=new, do_sample=False, eos_token_id=eos, pad_token_id=15)

    return run, calls


def test_low_level_steps_without_eos(monkeypatch):
    """No EOS id: every row advances one position per step through the fused
    append + decode, for max_new_tokens steps (paged_kv.py:840-985)."""
    run, calls = _fake_low_level(monkeypatch, [[1, 2], [3, 4], [5, 6]])
    out = run([10, 20], None, 3)
    assert out.tolist() == [[1, 3, 5], [2, 4, 6]]
    assert calls == [("fused", [11, 21]), ("fused", [12, 22]), ("fused", [13, 23])]


def test_low_level_steps_with_eos(monkeypatch):
    """Row 1 emits EOS (9) at step 1: from step 2 it keeps its length (append at
    the unchanged length, then decode over the others' new lengths) and
    re-emits input_ids[1, 0]; row 0 keeps advancing."""
    run, calls = _fake_low_level(monkeypatch, [[5, 6], [7, 9], [8, 10], [11, 12]])
    out = run([10, 20], 9, 4)
    assert out.tolist() == [[5, 7, 8, 11], [6, 9, 14, 14]]
    assert calls == [("fused", [11, 21]), ("fused", [12, 22]),
                     ("append", [12, 22]), ("decode", [13, 22]),
                     ("append", [13, 22]), ("decode", [14, 22])]


def test_low_level_stops_when_every_row_finished(monkeypatch):
    """Both rows emit EOS by step 1: the loop stops before step 2, whose column
    stays pad_token_id; row 0 re-emits input_ids[0, 0] at step 1."""
    run, calls = _fake_low_level(monkeypatch, [[9, 6], [1, 9], [2, 3]])
    out = run([10, 20], 9, 3)
    assert out.tolist() == [[9, 13, 15], [6, 9, 15]]
    assert [c[0] for c in calls] == ["fused", "append", "decode"]


# ----------------------------------------------------------------------- façade
def test_facade_routes_low_level(monkeypatch):
    seen = {}

    def fake_low(input_ids, **kw):
        seen.update(kw)
        return "low"

    monkeypatch.setattr(pkg, "_paged_kv_decode_low_level", fake_low)
    monkeypatch.setattr(pkg, "PAGED_KV_AVAILABLE", True)
    kw = {k: object() for k in ("k_cache", "v_cache", "block_tables", "context_lens", "qkv_proj_fn", "logits_fn")}
    assert pkg.paged_kv_decode(None, torch.zeros(1, 2), max_new_tokens=5, temperature=0.5, **kw) == "low"
    assert seen["max_new_tokens"] == 5 and seen["temperature"] == 0.5 and seen["do_sample"] is True
    assert seen["top_p"] == 1.0 and seen["pad_token_id"] is None and seen["eos_token_id"] is None


def test_facade_routes_model_and_left_trims(monkeypatch):
    seen = {}

    def fake_model(**kw):
        seen.update(kw)
        return "model"

    monkeypatch.setattr(pkg, "paged_kv_decode_model", fake_model)
    monkeypatch.setattr(pkg, "PAGED_KV_AVAILABLE", True)
    ids = torch.tensor([[0, 0, 5, 6], [0, 7, 8, 9]])
    mask = torch.tensor([[0, 0, 1, 1], [0, 1, 1, 1]])
    assert pkg.paged_kv_decode("m", ids, mask, max_new_tokens=3, do_sample=False, eos_token_id=2) == "model"
    assert seen["input_ids"].shape == (2, 3) and torch.equal(seen["input_ids"][1], torch.tensor([7, 8, 9]))
    assert seen["block_size"] == 16 and seen["pad_token_id"] == 0 and seen["do_sample"] is False
    assert seen["eos_token_id"] == 2 and seen["seed"] is None


def test_facade_raises_import_error_without_library(monkeypatch):
    monkeypatch.setattr(pkg, "PAGED_KV_AVAILABLE", False)
    with pytest.raises(ImportError):
        pkg.paged_kv_decode(None, torch.zeros(1, 2))


def test_trainer_flag_name_exported():
    assert pkg.TRITON_AVAILABLE is pkg.PAGED_KV_AVAILABLE


# --------------------------------------------------------------------- sampling
def test_greedy_sampling_is_argmax():
    logits = torch.randn(4, 50)
    assert torch.equal(paged_kv._sample_tokens(logits, False, 1.0, 1.0, None), logits.argmax(-1))
    assert torch.equal(paged_kv._sample_tokens(logits, True, 0.0, 1.0, None), logits.argmax(-1))


def test_top_p_keeps_smallest_nucleus():
    logits = torch.log(torch.tensor([[0.5, 0.3, 0.15, 0.05]]))
    # reference rule (paged_kv.py:424-433): drop sorted tokens whose cumulative mass exceeds top_p
    kept = paged_kv._apply_top_p(logits, 0.85)  # cumulative 0.5, 0.8, 0.95, 1.0
    assert torch.isfinite(kept[0, :2]).all() and torch.isinf(kept[0, 2:]).all()
    kept = paged_kv._apply_top_p(logits, 0.7)
    assert torch.isfinite(kept[0, :1]).all() and torch.isinf(kept[0, 1:]).all()
    assert torch.isfinite(paged_kv._apply_top_p(logits, 0.01)[0, 0])  # the top token always survives
    assert torch.isinf(paged_kv._apply_top_p(logits, 0.0)).all()
    assert torch.equal(paged_kv._apply_top_p(logits, 1.0), logits)


def test_seeded_sampling_is_reproducible():
    logits = torch.randn(8, 100)
    g1 = torch.Generator().manual_seed(3)
    g2 = torch.Generator().manual_seed(3)
    a = paged_kv._sample_tokens(logits, True, 0.7, 0.9, g1)
    b = paged_kv._sample_tokens(logits, True, 0.7, 0.9, g2)
    assert torch.equal(a, b)


# --------------------------------------------------------------------- page pool
def _pool(n=16, **kw):
    return KVPagePool(n, 2, 2, 4, 8, dtype=torch.float32, device="cpu", **kw)


def test_pool_alloc_free_and_exhaustion():
    pool = _pool()
    a = pool.alloc(10)
    assert len(set(a)) == 10 and pool.num_free == 6
    with pytest.raises(PoolExhausted):
        pool.alloc(7)
    pool.free(a[:4])
    assert pool.num_free == 10
    with pytest.raises(ValueError, match="double free"):
        pool.free([a[0]])


def test_pool_fork_refcounts():
    pool = _pool()
    a = pool.alloc(3)
    pool.fork(a)
    assert all(pool.refcount(p) == 2 for p in a)
    pool.free(a)
    assert pool.num_free == 13
    pool.free(a)
    assert pool.num_free == 16
    with pytest.raises(ValueError):
        pool.fork(a)


def test_pool_share_prefix_and_copy_on_write():
    pool = _pool(32)
    tables = pool.share_prefix(num_seqs=3, prefix_tokens=10, total_tokens=17)  # bs 4: 2 full shared pages
    assert all(len(t) == math.ceil(17 / 4) for t in tables)
    assert tables[0][:2] == tables[1][:2] == tables[2][:2]
    assert len({t[2] for t in tables}) == 3  # the partial prefix page is private
    assert pool.refcount(tables[0][0]) == 3
    pool.k[:, tables[0][2]] = 7.0
    pool.copy_prefix_tail(tables, 10)
    assert (pool.k[:, tables[2][2]] == 7.0).all()
    shared = tables[1][0]
    new = pool.make_private(tables[1], 0)
    assert new != shared and pool.refcount(shared) == 2 and tables[1][0] == new
    bt = pool.block_table(tables)
    assert bt.dtype == torch.int32 and bt.shape == (3, 5)


def test_pool_share_prompts_groups_rows():
    # rows 0, 2, 3 have one prompt, rows 1, 4 another; bs 4, prefix 10 -> 2 full shared pages per group
    groups = [0, 1, 0, 0, 1]
    need = KVPagePool.pages_needed_shared(groups, 10, 17, 4)
    assert need == 2 * 2 + 5 * (5 - 2)
    pool = _pool(need)
    tables, reps = pool.share_prompts(groups, prefix_tokens=10, total_tokens=17)
    assert reps == [0, 1] and pool.num_free == 0
    assert tables[0][:2] == tables[2][:2] == tables[3][:2] and tables[1][:2] == tables[4][:2]
    assert not set(tables[0][:2]) & set(tables[1][:2])
    assert pool.refcount(tables[0][0]) == 3 and pool.refcount(tables[1][0]) == 2
    private = [p for t in tables for p in t[2:]]
    assert len(set(private)) == len(private) == 15 and all(pool.refcount(p) == 1 for p in private)
    pool.k[:, tables[0][2]] = 3.0
    pool.v[:, tables[1][2]] = 5.0
    pool.copy_prefix_tails(tables, groups, 10)
    assert (pool.k[:, tables[2][2]] == 3.0).all() and (pool.k[:, tables[3][2]] == 3.0).all()
    assert (pool.v[:, tables[4][2]] == 5.0).all() and (pool.k[:, tables[4][2]] == 0.0).all()


def test_pool_share_prompts_without_repeats_is_private():
    pool = _pool(12)
    tables, reps = pool.share_prompts([0, 1, 2], prefix_tokens=8, total_tokens=13)
    assert reps == [0, 1, 2] and sorted(p for t in tables for p in t) == list(range(12))
    pool.copy_prefix_tails(tables, [0, 1, 2], 8)  # page-aligned prefix: nothing to copy


def test_prompt_groups_detects_repeated_prompts():
    ids = torch.tensor([[1, 2, 3], [4, 5, 6], [1, 2, 3], [1, 2, 3]])
    mask = torch.ones_like(ids)
    assert paged_kv._prompt_groups(ids, mask) == [0, 1, 0, 0]
    mask2 = mask.clone()
    mask2[2, 0] = 0  # same tokens, different padding: a different prompt
    assert paged_kv._prompt_groups(ids, mask2) == [0, 1, 2, 0]
    one = torch.tensor([[7, 8]]).expand(5, -1)
    assert paged_kv._prompt_groups(one, torch.ones(1, 2, dtype=torch.long).expand(5, -1)) == [0] * 5


def test_facade_return_prompt_layout(monkeypatch):
    seen = {}

    def fake_model(**kw):
        seen.update(kw)
        return torch.full((kw["input_ids"].shape[0], kw["max_new_tokens"]), 9, dtype=torch.int32)

    monkeypatch.setattr(pkg, "paged_kv_decode_model", fake_model)
    monkeypatch.setattr(pkg, "PAGED_KV_AVAILABLE", True)
    ids = torch.tensor([[0, 0, 5, 6], [0, 7, 8, 9]])
    mask = torch.tensor([[0, 0, 1, 1], [0, 1, 1, 1]])
    out = pkg.paged_kv_decode("m", ids, mask, max_new_tokens=3, return_prompt=True, share_prompt_pages=False)
    assert out.shape == (2, 7) and out.dtype == ids.dtype
    assert torch.equal(out[:, :4], ids) and (out[:, 4:] == 9).all()  # the trainer's outputs[j, prompt_len:]
    assert seen["share_prompt_pages"] is False and "return_prompt" not in seen
    assert pkg.paged_kv_decode("m", ids, mask, max_new_tokens=3).shape == (2, 3)
    assert seen["share_prompt_pages"] is True


# ---------------------------------------------------------------------- sharding
def test_lpt_assign_partitions_and_balances():
    import random

    rng = random.Random(0)
    costs = [rng.randint(1024, 8192) for _ in range(1024)]
    for world in (1, 2, 4, 8):
        parts = lpt_assign(costs, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(len(costs)))
        assert imbalance(costs, parts) < 1.01
    assert lpt_assign([5, 1], 4)[2:] == [[], []]
    assert shard_groups([3, 2, 1], 2, 0) == [0]


def test_sampling_oracle_keeps_the_reference_nucleus():
    """oracle.sample_top_p keeps exactly the tokens _apply_top_p (the reference rule,
    paged_kv.py:418-434) leaves finite, on fp32 logits without ties."""
    from oracle import oracle

    g = torch.Generator().manual_seed(2)
    logits = torch.randn(6, 300, generator=g) * 3
    for top_p in (0.3, 0.8, 0.97):
        kept = torch.isfinite(paged_kv._apply_top_p(logits / 0.7, top_p))
        # many uniforms per row: every token the oracle can return is in the nucleus,
        # and the sampled set covers the nucleus
        u = torch.linspace(0.0005, 0.9995, 2000)
        for b in range(logits.shape[0]):
            toks, _, _ = oracle.sample_top_p(logits[b:b + 1].repeat(len(u), 1), 0.7, top_p, u)
            assert set(toks.tolist()) <= set(kept[b].nonzero().flatten().tolist())
            assert set(toks.tolist()) == set(kept[b].nonzero().flatten().tolist()) or kept[b].sum() > 50
