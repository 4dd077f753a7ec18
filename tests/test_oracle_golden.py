"""Pin the CPU oracle to the reference: golden vectors made by the reference's own kernels.

tests/golden/*.npz hold outputs of the reference Triton kernels
(src/triton_kernels/paged_kv.py:63-319, run under the Triton interpreter by
tests/golden/make_golden.py). Here the oracle must reproduce them: the
append and prompt scatter byte for byte (SHA-256 of the caches), the decode
within 1e-5 max-abs. The CUDA tests then compare against this oracle.
"""

from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest
import torch

import cases
from conftest import GOLDEN, load_golden
from oracle import oracle

RAW = {torch.float32: torch.int32, torch.bfloat16: torch.int16, torch.float16: torch.int16}


def _sha(*tensors: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(np.ascontiguousarray(t.contiguous().view(RAW[t.dtype]).numpy()).tobytes())
    return h.hexdigest()


@pytest.fixture(scope="module", autouse=True)
def _built():
    oracle.build()


@pytest.mark.parametrize("name", [c["name"] for c in cases.CASES])
def test_inputs_regenerate_exactly(name):
    _, meta = load_golden(name)
    assert cases.inputs_sha(cases.make_inputs(cases.BY_NAME[name])) == meta["inputs_sha"]


@pytest.mark.parametrize("name", [c["name"] for c in cases.CASES])
def test_oracle_matches_reference_kernels(name):
    case = cases.BY_NAME[name]
    ref_out, meta = load_golden(name)
    t = cases.to_torch(cases.make_inputs(case), case["dtype"])
    ctx = t["context_lens"]
    if case["append"]:
        oracle.append(t["k_new"], t["v_new"], t["k_cache"], t["v_cache"], t["block_tables"], ctx)
        ctx = ctx + 1
    # append is bit-exact against the reference update kernel
    assert _sha(t["k_cache"], t["v_cache"]) == meta["cache_after_append_sha"]
    out = oracle.decode(t["q"], t["k_cache"], t["v_cache"], t["block_tables"], ctx)
    np.testing.assert_allclose(out.numpy(), ref_out, rtol=0, atol=1e-5)
    out_np = oracle.decode_numpy(t["q"], t["k_cache"], t["v_cache"], t["block_tables"], ctx)
    np.testing.assert_allclose(out_np, ref_out, rtol=0, atol=1e-5)


@pytest.mark.parametrize("name", [c["name"] for c in cases.CASES if c.get("prompt_steps")])
def test_oracle_prompt_scatter_matches_reference(name):
    case = cases.BY_NAME[name]
    _, meta = load_golden(name)
    t = cases.to_torch(cases.make_inputs(case), case["dtype"])
    kc = torch.zeros_like(t["k_cache"])
    vc = torch.zeros_like(t["v_cache"])
    oracle.append_prompt(t["prompt_k"], t["prompt_v"], kc, vc, t["block_tables"])
    assert _sha(kc, vc) == meta["prompt_cache_sha"]


def test_oracle_gather_round_trip():
    case = cases.BY_NAME["bf16_prompt_d128"]
    t = cases.to_torch(cases.make_inputs(case), case["dtype"])
    kc = torch.zeros_like(t["k_cache"])
    vc = torch.zeros_like(t["v_cache"])
    oracle.append_prompt(t["prompt_k"], t["prompt_v"], kc, vc, t["block_tables"])
    steps = case["prompt_steps"]
    k, v = oracle.gather(kc, vc, t["block_tables"], torch.full((case["batch"],), steps, dtype=torch.int32))
    assert torch.equal(k[:, :, :steps].view(torch.int16), t["prompt_k"].view(torch.int16))
    assert torch.equal(v[:, :, :steps].view(torch.int16), t["prompt_v"].view(torch.int16))
    assert not k[:, :, steps:].view(torch.int16).any()


def test_oracle_empty_context_is_zero():
    q = torch.randn(2, 4, 32)
    kc = torch.randn(4, 2, 16, 32)
    bt = torch.arange(4, dtype=torch.int32).reshape(2, 2)
    out = oracle.decode(q, kc, kc.clone(), bt, torch.zeros(2, dtype=torch.int32))
    assert not out.any()


def test_oracle_threads_do_not_change_result():
    case = cases.BY_NAME["bf16_qwen7b_g7"]
    t = cases.to_torch(cases.make_inputs(case), case["dtype"])
    a = oracle.decode(t["q"], t["k_cache"], t["v_cache"], t["block_tables"], t["context_lens"], nthreads=1)
    b = oracle.decode(t["q"], t["k_cache"], t["v_cache"], t["block_tables"], t["context_lens"], nthreads=7)
    assert torch.equal(a, b)


def test_planted_mistake_is_caught():
    """A wrong scale in the oracle must fail the golden comparison (the check has teeth)."""
    case = cases.BY_NAME["config1_fp32"]
    ref_out, _ = load_golden("config1_fp32")
    t = cases.to_torch(cases.make_inputs(case), case["dtype"])
    oracle.append(t["k_new"], t["v_new"], t["k_cache"], t["v_cache"], t["block_tables"], t["context_lens"])
    bad = oracle.decode(t["q"], t["k_cache"], t["v_cache"], t["block_tables"], t["context_lens"] + 1,
                        scale=1.01 / np.sqrt(case["head_dim"]))
    assert np.abs(bad.numpy() - ref_out).max() > 1e-5


# ------------------------------------------------------------ sampling nucleus
# The reference computes its nucleus in the logits dtype: probabilities rounded to
# it and an fp32 running sum rounded to it (torch's softmax / cumsum on CPU), so its
# cut can sit a rounding step away from the exact rule's; and its default sort is
# not stable, so among tokens with equal scaled logits at the cut the kept ones
# are not defined. Where the two rules differ, the cut must therefore fall within
# the rounding band of the differing token's group: top_p in [lo - delta, hi + delta],
# lo = the exact mass above the token's scaled value, hi = lo + the group's mass.
NUCLEUS_DELTA = {"float32": 1e-5, "bfloat16": 2.0 ** -8, "float16": 2.0 ** -10}


def _sampling_fixture(name: str):
    data = np.load(GOLDEN / f"sampling_{name}.npz")
    return data["kept"], json.loads(str(data["meta"]))


@pytest.mark.parametrize("name", [c["name"] for c in cases.SAMPLING_CASES])
def test_oracle_nucleus_matches_the_reference_apply_top_p(name):
    case = next(c for c in cases.SAMPLING_CASES if c["name"] == name)
    kept_ref_packed, meta = _sampling_fixture(name)
    logits_np = cases.make_sampling_logits(case)
    assert hashlib.sha256(np.ascontiguousarray(logits_np).tobytes()).hexdigest() == meta["logits_sha"]
    logits = torch.from_numpy(logits_np).to(getattr(torch, case["dtype"]))
    rows, vocab = logits.shape
    delta = NUCLEUS_DELTA[case["dtype"]]
    identical = 0
    for k, (temperature, top_p) in enumerate(cases.SAMPLING_PARAMS):
        kept_ref = np.unpackbits(kept_ref_packed[k], axis=-1, count=vocab).astype(bool)
        kept, scaled, p = oracle.nucleus(logits, temperature, top_p)
        for b in range(rows):
            diff = np.nonzero(kept[b] != kept_ref[b])[0]
            if diff.size == 0:
                identical += 1
                continue
            for t in diff:
                v = scaled[b, t]
                lo = float(p[b, scaled[b] > v].sum())
                hi = lo + float(p[b, scaled[b] == v].sum())
                assert lo - delta <= top_p <= hi + delta, (name, temperature, top_p, b, int(t), lo, hi)
    # rounding only matters near the cut: rows of few ties mostly agree token
    # for token (bf16 rows of a large vocabulary tie at the cut almost always)
    if case["kind"] == "normal" and vocab <= 1000:
        assert identical >= rows * len(cases.SAMPLING_PARAMS) // 2, identical


def test_oracle_nucleus_fp32_rows_agree_exactly_with_the_reference():
    """fp32 logits without ties: the exact rule and the reference's fp32 rule
    keep the same tokens on every row of the fixture."""
    case = next(c for c in cases.SAMPLING_CASES if c["name"] == "f32_v1000")
    kept_ref_packed, _ = _sampling_fixture(case["name"])
    logits = torch.from_numpy(cases.make_sampling_logits(case))
    for k, (temperature, top_p) in enumerate(cases.SAMPLING_PARAMS):
        kept_ref = np.unpackbits(kept_ref_packed[k], axis=-1, count=logits.shape[1]).astype(bool)
        kept, _, _ = oracle.nucleus(logits, temperature, top_p)
        assert np.array_equal(kept, kept_ref), (temperature, top_p)


# ------------------------------------------------------------ RMSNorm
@pytest.mark.parametrize("name", [c["name"] for c in cases.RMSNORM_CASES])
def test_oracle_rmsnorm_matches_the_reference_kernel(name):
    case = next(c for c in cases.RMSNORM_CASES if c["name"] == name)
    ref_bits, meta = load_golden(name)
    inp = cases.make_rmsnorm_inputs(case)
    assert cases.inputs_sha(inp) == meta["inputs_sha"]
    x = torch.from_numpy(inp["x"]).to(torch.bfloat16)
    w = torch.from_numpy(inp["weight"]).to(torch.bfloat16)
    # The fixture comes from Triton's interpreter, whose fp32 -> bf16 cast rounds
    # toward zero (compiled Triton rounds to nearest even); with that rounding the
    # restatement reproduces the reference kernel bit for bit, which pins every
    # other step (sum of squares, mean, eps, rsqrt, the two products).
    got = oracle.rmsnorm(x, w, case["eps"], cast_rounding="rtz")
    ref = torch.from_numpy(ref_bits).view(torch.bfloat16)
    assert torch.equal(got, ref)
