"""Pin the CPU oracle to the reference: golden vectors made by the reference's own kernels.

tests/golden/*.npz hold outputs of the reference Triton kernels
(src/triton_kernels/paged_kv.py:63-319, run under the Triton interpreter by
tests/golden/make_golden.py). Here the oracle must reproduce them: the
append and prompt scatter byte for byte (SHA-256 of the caches), the decode
within 1e-5 max-abs. The CUDA tests then compare against this oracle.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

import cases
from conftest import load_golden
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
