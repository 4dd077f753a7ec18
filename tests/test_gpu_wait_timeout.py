"""The decode kernel's bounded device waits run out, report, and return.

Every mbarrier wait in the tensor-core decode kernel gives up after a bounded
number of polls, ORs PKV_DEV_WAIT_TIMEOUT into the caller's status word and
lets the kernel return, so a lost pipeline element can never hang the GPU.
The test flag PKV_DECODE_TEST_WAIT_TIMEOUT shortens every bound to 4096 polls
and makes the first CTA's producer withhold one element: its consumer warp
waits for an element that never comes, the other warps then wait at the unit
barrier for that warp, and the producer waits for a ring slot the warp never
frees. Nothing faults or traps; the waits simply run out. The test checks
that the launch ends promptly, that the status word carries the timeout bit,
and that a normal decode on the same stream right after it, with a new plan
(a launch that timed out may leave a split's merge counter mid-count, so its
plan is not reused), is correct: the context is still usable.
"""

from __future__ import annotations

import math
import time

import pytest
import torch

from conftest import ATOL
from grpo_training_engine_b200 import _lib, decode_kernel_kind, paged_attention_decode, plan_decode
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _case(seed, batch=64, hq=12, hkv=2, d=128, bs=16):
    g = torch.Generator().manual_seed(seed)
    ctxs = torch.randint(100, 3000, (batch,), generator=g)
    max_blocks = math.ceil(int(ctxs.max()) / bs) + 1
    nb = batch * max_blocks
    bt = torch.randperm(nb, generator=g).reshape(batch, max_blocks).int()
    q = torch.randn(batch, hq, d, generator=g).to(torch.bfloat16)
    kc = torch.randn(nb, hkv, bs, d, generator=g).to(torch.bfloat16)
    vc = torch.randn(nb, hkv, bs, d, generator=g).to(torch.bfloat16)
    return q, kc, vc, bt, ctxs.int()


@pytest.mark.parametrize("pages_per_split", [0, 16])
def test_wait_timeout_is_reported_and_the_context_stays_usable(pages_per_split):
    q, kc, vc, bt, ctx = _case(7)
    qd, kd, vd, btd, ctxd = (t.to(DEV) for t in (q, kc, vc, bt, ctx))
    assert decode_kernel_kind(qd, kd) == "tensor_core"
    B, hq, d = q.shape
    nb, hkv, bs, _ = kc.shape
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    plan = plan_decode(ctxd, hq, hkv, d, bs, bt.shape[1], pages_per_split=pages_per_split, status=status)
    out = torch.empty(B, hq, d, dtype=torch.float32, device=DEV)
    ws = plan.workspace
    i64 = _lib.i64_array
    torch.cuda.synchronize()
    t0 = time.monotonic()
    rc = _lib.load().pkv_decode_run(
        qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), btd.data_ptr(), plan.context_lens.data_ptr(), out.data_ptr(),
        B, hq, hkv, d, bs, nb, bt.shape[1], i64(qd.stride()), i64(kd.stride()), i64(btd.stride()),
        i64(out.stride()), _lib.DTYPE_BF16, _lib.DTYPE_BF16, 1.0 / math.sqrt(d), plan.pages_per_split,
        _lib.DECODE_TEST_WAIT_TIMEOUT, ws.data_ptr(), ws.numel(), status.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_detail()
    torch.cuda.synchronize()
    elapsed = time.monotonic() - t0
    assert elapsed < 10.0, elapsed  # the short bounds end the launch in milliseconds
    assert int(status.item()) & _lib.DEV_WAIT_TIMEOUT

    # the same stream, a new plan in the same workspace: a normal decode is correct
    status.zero_()
    plan = plan_decode(ctxd, hq, hkv, d, bs, bt.shape[1], pages_per_split=pages_per_split, workspace=ws,
                       status=status)
    out2 = paged_attention_decode(qd, kd, vd, btd, ctxd, plan=plan, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = oracle.decode(q, kc, vc, bt, ctx)
    assert float((out2.cpu() - ref).abs().max()) <= ATOL["bfloat16"]
