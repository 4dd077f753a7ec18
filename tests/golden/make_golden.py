"""Generate tests/golden/*.npz by running the REFERENCE's own paged-KV kernels.

Run in a container that has the reference checkout (it is not needed by the
tests themselves):

    python tests/golden/make_golden.py /path/to/grpo-training-engine

It imports src/triton_kernels/paged_kv.py from that checkout and launches
its raw Triton kernels ``_paged_kv_update_kernel`` and
``_paged_attention_decode_kernel`` on CPU tensors under the Triton
interpreter (TRITON_INTERPRET=1), with the argument lists and launch
heuristics of the reference's own drivers (paged_kv.py:730-783, 914-969).
The reference kernel indexes cache head = query head (grid (B, H)), so a
grouped-query case is run on a cache replicated to Hq heads, exactly as the
reference model path does with repeat_kv (paged_kv.py:574-575, 723-724);
the fixture stores the un-replicated (Hkv) cache contents.

Inputs are drawn from numpy's legacy RandomState (a stream frozen across
numpy versions) so the tests regenerate them from the seed; each fixture
stores a SHA-256 of its inputs to catch any drift, the reference outputs,
and SHA-256 digests of the caches after the reference's appends.

Two more parts pin the steps around the decode in the rollout step:
  sampling: the reference's _apply_top_p (paged_kv.py:418-434) on rows of
            logits scaled as _sample_tokens scales them (paged_kv.py:437-450),
            for every (temperature, top_p) of cases.SAMPLING_PARAMS; the
            fixture stores the kept-token masks (sampling_<case>.npz);
  rmsnorm:  the reference's fused_rmsnorm (fused_ops.py:118-148, Triton kernel
            :34-77, under the interpreter) on bf16 rows; the fixture stores the
            output bits (rmsnorm_<case>.npz).

    python tests/golden/make_golden.py <reference checkout> [--only decode,sampling,rmsnorm]

`--time` instead prints the seconds per call of the reference's append + decode
kernels on the config-1 case under the interpreter (the reference's own code on
the host CPU):

    python tests/golden/make_golden.py <reference checkout> --time
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases  # noqa: E402  (tests/golden/cases.py: the case list and input generator)


def _sha(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def sampling_fixtures(ref, torch) -> None:
    for case in cases.SAMPLING_CASES:
        logits = torch.from_numpy(cases.make_sampling_logits(case)).to(getattr(torch, case["dtype"]))
        masks = []
        for temperature, top_p in cases.SAMPLING_PARAMS:
            scaled = logits / max(temperature, 1e-6)  # _sample_tokens (paged_kv.py:446)
            kept = torch.isfinite(ref._apply_top_p(scaled, top_p))
            masks.append(np.packbits(kept.numpy(), axis=-1))
        meta = {
            "case": case["name"],
            "params": cases.SAMPLING_PARAMS,
            "logits_sha": _sha(cases.make_sampling_logits(case)),
            "generator": "reference _apply_top_p (torch, CPU) on logits / max(T, 1e-6)",
        }
        np.savez_compressed(HERE / f"sampling_{case['name']}.npz", kept=np.stack(masks), meta=json.dumps(meta))
        print("sampling", case["name"], [int(np.unpackbits(m, axis=-1).sum()) for m in masks])


def rmsnorm_fixtures(torch) -> None:
    from src.triton_kernels import fused_ops  # the reference module

    # The rollout step runs the kernel on bf16 rows and a bf16 weight. Triton
    # 3.6's interpreter multiplies two bf16 operands wrongly (the kernel's
    # `normed * w`, fused_ops.py:74, comes out as garbage; a bf16 x fp32 product
    # is right), so the kernel is run on fp32 tensors that hold the bf16 values:
    # every step is the same (the loads are cast to fp32 anyway, `normed` is
    # still rounded to bf16 by the kernel's own cast, :73), and the product of
    # two bf16 values is exact in fp32, so rounding the fp32 output to bf16 gives
    # the bf16 kernel's result (a bf16 product correctly rounded).
    for case in cases.RMSNORM_CASES:
        inp = cases.make_rmsnorm_inputs(case)
        x = torch.from_numpy(inp["x"]).to(torch.bfloat16).float()
        w = torch.from_numpy(inp["weight"]).to(torch.bfloat16).float()
        y = fused_ops.fused_rmsnorm(x[:, None, :], w, case["eps"])[:, 0, :].to(torch.bfloat16)
        meta = {
            "case": case["name"],
            "inputs_sha": cases.inputs_sha(inp),
            "generator": "reference fused_rmsnorm (Triton kernel under TRITON_INTERPRET=1) on fp32 tensors "
                         "holding the bf16 values, output rounded to bf16",
        }
        np.savez_compressed(HERE / f"{case['name']}.npz", out=y.contiguous().view(torch.int16).numpy(),
                            meta=json.dumps(meta))
        print(case["name"], tuple(y.shape))


def reference_append_decode(ref, torch, case: dict, t: dict):
    """One layer of the reference's step on a case: its update kernel appends the
    new token (when the case has one), then its decode kernel attends over the
    post-append lengths, with the launch arguments and heuristics of the
    reference drivers (paged_kv.py:730-783). Returns the head-replicated caches,
    the block tables, the fp32 output and the head-dim block used."""
    G = case["hq"] // case["hkv"]
    B, bs = case["batch"], case["block_size"]
    D = case["head_dim"]
    # replicate the cache to query heads (reference model-path layout)
    kc = t["k_cache"].repeat_interleave(G, dim=1).contiguous()
    vc = t["v_cache"].repeat_interleave(G, dim=1).contiguous()
    bt = t["block_tables"]
    ctx_pre = t["context_lens"]
    block_d = ref._select_block_d(D)
    max_context = bt.shape[1] * bs
    if case["append"]:
        k_new = t["k_new"].repeat_interleave(G, dim=1).contiguous()
        v_new = t["v_new"].repeat_interleave(G, dim=1).contiguous()
        ref._paged_kv_update_kernel[(B, case["hq"])](
            k_new, v_new, kc, vc, bt, ctx_pre,
            k_new.stride(0), k_new.stride(1), k_new.stride(2),
            kc.stride(0), kc.stride(1), kc.stride(2), kc.stride(3),
            bt.stride(0), bt.stride(1), bs,
            D=D, BLOCK_D=block_d, num_warps=ref._select_num_warps_update(D), num_stages=1,
        )
        ctx = ctx_pre + 1
    else:
        ctx = ctx_pre
    q = t["q"]
    out = torch.empty((B, case["hq"], D), dtype=torch.float32)
    block_ctx = ref._select_block_ctx(max_context)
    ref._paged_attention_decode_kernel[(B, case["hq"])](
        q, kc, vc, bt, ctx, out,
        q.stride(0), q.stride(1), q.stride(2),
        kc.stride(0), kc.stride(1), kc.stride(2), kc.stride(3),
        bt.stride(0), bt.stride(1),
        out.stride(0), out.stride(1), out.stride(2),
        bs, 1.0 / np.sqrt(D),
        D=D, BLOCK_CTX=block_ctx, BLOCK_D=block_d, MAX_CONTEXT=max_context,
        num_warps=ref._select_num_warps_decode(block_d, block_ctx), num_stages=1,
    )
    return kc, vc, bt, out, block_d


def time_reference(ref_root: str, calls: int = 3) -> None:
    """Seconds per call of the reference's append + decode kernels on the
    config-1 case (1.5B head geometry, fp32, contexts 37/128/300/511 + 1) under
    the Triton interpreter on this machine's CPU: the reference's own code on
    the host, stated beside the CPU baselines."""
    import time

    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, ref_root)
    import torch
    from src.triton_kernels import paged_kv as ref  # the reference module

    case = cases.BY_NAME["config1_fp32"]
    times = []
    for _ in range(calls + 1):  # the first call compiles nothing but warms the interpreter's caches
        t = cases.to_torch(cases.make_inputs(case), case["dtype"])
        t0 = time.perf_counter()
        reference_append_decode(ref, torch, case, t)
        times.append(time.perf_counter() - t0)
    print(json.dumps({"case": case["name"], "seconds_per_call": [round(x, 2) for x in times[1:]],
                      "first_call_s": round(times[0], 2), "cpus": os.cpu_count()}))


def main(ref_root: str, parts=("decode", "sampling", "rmsnorm")) -> None:
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, ref_root)
    import torch
    from src.triton_kernels import paged_kv as ref  # the reference module

    if "sampling" in parts:
        sampling_fixtures(ref, torch)
    if "rmsnorm" in parts:
        rmsnorm_fixtures(torch)
    for case in (cases.CASES if "decode" in parts else []):
        inp = cases.make_inputs(case)
        t = cases.to_torch(inp, case["dtype"])
        G = case["hq"] // case["hkv"]
        B, bs = case["batch"], case["block_size"]
        D = case["head_dim"]
        kc, vc, bt, out, block_d = reference_append_decode(ref, torch, case, t)
        # the un-replicated cache after the reference append: head kvh*G of the replica
        kc_gqa = kc[:, ::G].contiguous()
        vc_gqa = vc[:, ::G].contiguous()
        raw = {torch.float32: torch.int32, torch.bfloat16: torch.int16, torch.float16: torch.int16}[kc.dtype]
        extra = {}
        if case.get("prompt_steps"):
            # position-by-position prompt writes with the reference update kernel:
            # the scatter rule of _prefill_paged_cache (paged_kv.py:576-586)
            pk = t["prompt_k"].repeat_interleave(G, dim=1)
            pv = t["prompt_v"].repeat_interleave(G, dim=1)
            pkc = torch.zeros_like(kc)
            pvc = torch.zeros_like(vc)
            for step in range(case["prompt_steps"]):
                kn = pk[:, :, step, :].contiguous()
                vn = pv[:, :, step, :].contiguous()
                pos = torch.full((B,), step, dtype=torch.int32)
                ref._paged_kv_update_kernel[(B, case["hq"])](
                    kn, vn, pkc, pvc, bt, pos,
                    kn.stride(0), kn.stride(1), kn.stride(2),
                    pkc.stride(0), pkc.stride(1), pkc.stride(2), pkc.stride(3),
                    bt.stride(0), bt.stride(1), bs,
                    D=D, BLOCK_D=block_d, num_warps=ref._select_num_warps_update(D), num_stages=1,
                )
            extra["prompt_cache_sha"] = _sha(pkc[:, ::G].contiguous().view(raw).numpy(),
                                             pvc[:, ::G].contiguous().view(raw).numpy())
        meta = {
            "case": case["name"],
            "inputs_sha": cases.inputs_sha(inp),
            "cache_after_append_sha": _sha(kc_gqa.view(raw).numpy(), vc_gqa.view(raw).numpy()),
            "generator": "reference Triton kernels under TRITON_INTERPRET=1",
            **extra,
        }
        np.savez_compressed(HERE / f"{case['name']}.npz", out=out.numpy(), meta=json.dumps(meta))
        print(case["name"], out.shape, float(out.abs().max()))


if __name__ == "__main__":
    args = sys.argv[1:]
    parts = ("decode", "sampling", "rmsnorm")
    if "--time" in args:
        args.remove("--time")
        time_reference(args[0])
        sys.exit(0)
    if "--only" in args:
        i = args.index("--only")
        parts = tuple(args[i + 1].split(","))
        del args[i:i + 2]
    if len(args) != 1:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout> [--only decode,sampling,rmsnorm] | --time")
    main(args[0], parts)
