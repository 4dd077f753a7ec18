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


def main(ref_root: str) -> None:
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, ref_root)
    import torch
    from src.triton_kernels import paged_kv as ref  # the reference module

    for case in cases.CASES:
        inp = cases.make_inputs(case)
        t = cases.to_torch(inp, case["dtype"])
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
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout>")
    main(sys.argv[1])
