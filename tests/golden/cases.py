"""Golden-vector cases: geometry, seeds and the deterministic input generator.

Shared by make_golden.py (which runs the reference kernels on these inputs)
and by the tests (which regenerate the same inputs and compare against the
stored reference outputs). Inputs come from numpy's legacy RandomState, whose
stream is frozen across numpy versions; ``inputs_sha`` lets a test prove it
regenerated exactly the inputs the fixture was made from.
"""

from __future__ import annotations

import hashlib

import numpy as np

CASES = [
    # 1.5B geometry, fp32, ctx {37,128,300,511} + 1 append,
    # 256-page pool, block tables = seeded shuffle of free page ids.
    dict(name="config1_fp32", seed=1, batch=4, hq=12, hkv=2, head_dim=128, block_size=16,
         num_blocks=256, max_blocks=32, ctx=[37, 128, 300, 511], dtype="float32", append=True),
    # grouped-query bf16, head_dim 64, includes an empty pre-append context
    dict(name="bf16_gqa_d64", seed=2, batch=3, hq=8, hkv=2, head_dim=64, block_size=16,
         num_blocks=40, max_blocks=8, ctx=[0, 17, 100], dtype="bfloat16", append=True),
    # Qwen2.5-7B head geometry (28 q / 4 kv heads), bf16
    dict(name="bf16_qwen7b_g7", seed=3, batch=2, hq=28, hkv=4, head_dim=128, block_size=16,
         num_blocks=100, max_blocks=48, ctx=[255, 700], dtype="bfloat16", append=True),
    # the reference test geometry (tests/test_triton_performance.py:144-150): H=2, D=8, bs=4
    dict(name="bf16_tiny_bs4", seed=4, batch=2, hq=2, hkv=2, head_dim=8, block_size=4,
         num_blocks=12, max_blocks=6, ctx=[2, 9], dtype="bfloat16", append=True, prompt_steps=10),
    # decode-only edge lengths: empty, one token, exactly one page, page + 1, full table
    dict(name="fp32_edges", seed=5, batch=5, hq=4, hkv=4, head_dim=32, block_size=16,
         num_blocks=24, max_blocks=4, ctx=[0, 1, 16, 17, 64], dtype="float32", append=False),
    # config-2 head geometry prompt write (40 positions) + append, 12q/2kv, bf16
    dict(name="bf16_prompt_d128", seed=6, batch=2, hq=12, hkv=2, head_dim=128, block_size=16,
         num_blocks=16, max_blocks=8, ctx=[40, 40], dtype="bfloat16", append=True, prompt_steps=40),
    # fp16 multi-query (one kv head for four query heads)
    dict(name="f16_mqa", seed=7, batch=2, hq=4, hkv=1, head_dim=128, block_size=16,
         num_blocks=20, max_blocks=10, ctx=[50, 150], dtype="float16", append=True),
]

BY_NAME = {c["name"]: c for c in CASES}


def make_inputs(case: dict) -> dict[str, np.ndarray]:
    rs = np.random.RandomState(case["seed"])
    B, hq, hkv, D = case["batch"], case["hq"], case["hkv"], case["head_dim"]
    nb, bs, mb = case["num_blocks"], case["block_size"], case["max_blocks"]
    perm = rs.permutation(nb)
    out = {
        "block_tables": perm[: B * mb].reshape(B, mb).astype(np.int32),
        "context_lens": np.asarray(case["ctx"], dtype=np.int32),
        "q": rs.standard_normal((B, hq, D)).astype(np.float32),
        "k_cache": rs.standard_normal((nb, hkv, bs, D)).astype(np.float32),
        "v_cache": rs.standard_normal((nb, hkv, bs, D)).astype(np.float32),
        "k_new": rs.standard_normal((B, hkv, D)).astype(np.float32),
        "v_new": rs.standard_normal((B, hkv, D)).astype(np.float32),
    }
    steps = case.get("prompt_steps", 0)
    if steps:
        out["prompt_k"] = rs.standard_normal((B, hkv, steps, D)).astype(np.float32)
        out["prompt_v"] = rs.standard_normal((B, hkv, steps, D)).astype(np.float32)
    return out


def inputs_sha(inp: dict[str, np.ndarray]) -> str:
    h = hashlib.sha256()
    for key in sorted(inp):
        h.update(key.encode())
        h.update(np.ascontiguousarray(inp[key]).tobytes())
    return h.hexdigest()


def to_torch(inp: dict[str, np.ndarray], dtype: str, device="cpu") -> dict:
    """Torch tensors of the inputs; float arrays cast (round-to-nearest-even) to `dtype`."""
    import torch

    dt = getattr(torch, dtype)
    res = {}
    for key, arr in inp.items():
        t = torch.from_numpy(arr)
        if arr.dtype == np.float32:
            t = t.to(dt)
        res[key] = t.to(device)
    return res


# ---------------------------------------------------------------- sampling nucleus
# Rows of logits for the reference's _apply_top_p (src/triton_kernels/paged_kv.py:418-434),
# applied as _sample_tokens applies it (paged_kv.py:437-450): scaled = logits / max(T, 1e-6)
# in the logits dtype. kind: "normal" N(0,1) * scale; "coarse": rounded to multiples of
# `step` (many equal values, ties at the cut); "peaked": one dominant token.
SAMPLING_CASES = [
    dict(name="f32_v1000", seed=21, rows=6, vocab=1000, dtype="float32", kind="normal", scale=3.0),
    dict(name="bf16_v1000", seed=22, rows=6, vocab=1000, dtype="bfloat16", kind="normal", scale=3.0),
    dict(name="f16_v1000", seed=23, rows=4, vocab=1000, dtype="float16", kind="normal", scale=3.0),
    dict(name="bf16_coarse_v5000", seed=24, rows=4, vocab=5000, dtype="bfloat16", kind="coarse", scale=2.0,
         step=0.5),
    dict(name="bf16_peaked_v3000", seed=25, rows=3, vocab=3000, dtype="bfloat16", kind="peaked", scale=1.0),
    dict(name="bf16_v151936", seed=26, rows=2, vocab=151936, dtype="bfloat16", kind="normal", scale=3.0),
]
# (temperature, top_p) pairs applied to every row
SAMPLING_PARAMS = [(0.7, 0.9), (1.0, 0.5), (0.5, 0.95), (1.3, 0.3)]


def make_sampling_logits(case: dict) -> np.ndarray:
    """fp32 [rows, vocab]; the tests and the generator cast it to case["dtype"]."""
    rs = np.random.RandomState(case["seed"])
    x = rs.standard_normal((case["rows"], case["vocab"])).astype(np.float32) * np.float32(case["scale"])
    if case["kind"] == "coarse":
        x = (np.round(x / case["step"]) * case["step"]).astype(np.float32)
    elif case["kind"] == "peaked":
        hot = rs.randint(0, case["vocab"], size=case["rows"])
        x[np.arange(case["rows"]), hot] += np.float32(12.0)
    return x


# ---------------------------------------------------------------- RMSNorm
# Rows for the reference's fused_rmsnorm (src/triton_kernels/fused_ops.py:118-148, kernel
# :34-77), bf16 x [rows, hidden] and weight [hidden], eps 1e-6: the hidden sizes of the
# 1.5B (1536) and 7B (3584) geometries and a short odd-sized row.
RMSNORM_CASES = [
    dict(name="rmsnorm_1536", seed=31, rows=16, hidden=1536, eps=1e-6),
    dict(name="rmsnorm_3584", seed=32, rows=8, hidden=3584, eps=1e-6),
    dict(name="rmsnorm_104", seed=33, rows=8, hidden=104, eps=1e-6),
]


def make_rmsnorm_inputs(case: dict) -> dict[str, np.ndarray]:
    rs = np.random.RandomState(case["seed"])
    rows, hidden = case["rows"], case["hidden"]
    x = rs.standard_normal((rows, hidden)).astype(np.float32) * np.float32(3.0)
    x[rows // 2:] *= np.float32(40.0)  # large activations too
    w = (np.float32(1.0) + np.float32(0.1) * rs.standard_normal(hidden)).astype(np.float32)
    return {"x": x, "weight": w}
