"""pkv_decode_noalloc: the decode entry point that allocates nothing.

Some callers cannot allocate device memory themselves — an FFI host that only
hands the library the tensors it owns, or a process whose GPU memory is held by
another framework's allocator. For them pkv_decode_noalloc takes no workspace
and uses a fixed scratch array built into libpkv.so instead. These tests call
it through the C ABI and check it against pkv_decode (with a workspace the test
allocates) on two calls in a row with different data, so a call that silently
reused the previous call's scratch contents would be caught. The file runs
last so that a stop-at-first-failure run has already run everything else.
"""

from __future__ import annotations

import ctypes as C
import math

import pytest
import torch

from conftest import ATOL
from grpo_training_engine_b200 import _lib, decode_workspace_bytes

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
DT = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}


def _case(seed, batch, hq, hkv, d, bs, ctxs, dtype):
    g = torch.Generator().manual_seed(seed)
    max_blocks = max(math.ceil(c / bs) for c in ctxs) + 1
    nb = batch * max_blocks + 3
    bt = torch.randperm(nb, generator=g)[: batch * max_blocks].reshape(batch, max_blocks).int()
    q = torch.randn(batch, hq, d, generator=g).to(dtype)
    kc = torch.randn(nb, hkv, bs, d, generator=g).to(dtype)
    vc = torch.randn(nb, hkv, bs, d, generator=g).to(dtype)
    ctx = torch.tensor(ctxs, dtype=torch.int32)
    return [t.to(DEV) for t in (q, kc, vc, bt, ctx)]


def _args(q, kc, vc, bt, ctx, out, pages_per_split, flags):
    batch, hq, d = q.shape
    nb, hkv, bs, _ = kc.shape
    i64 = _lib.i64_array
    head = [q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), ctx.data_ptr(), out.data_ptr(),
            batch, hq, hkv, d, bs, nb, bt.shape[1], i64(q.stride()), i64(kc.stride()), i64(bt.stride()),
            i64(out.stride()), DT[q.dtype], DT[kc.dtype], 1.0 / math.sqrt(d), pages_per_split, flags]
    return head


def _with_workspace(q, kc, vc, bt, ctx, pages_per_split=0, flags=0):
    """The existing entry point, pkv_decode, with a workspace allocated here."""
    out = torch.empty(q.shape, dtype=torch.float32, device=DEV)
    ws = torch.empty(decode_workspace_bytes(q.shape[0], q.shape[1], kc.shape[1], q.shape[2], bt.shape[1],
                                            pages_per_split), dtype=torch.uint8, device=DEV)
    rc = _lib.load().pkv_decode(*_args(q, kc, vc, bt, ctx, out, pages_per_split, flags), ws.data_ptr(),
                                ws.numel(), None, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_detail()
    return out


def _no_alloc(q, kc, vc, bt, ctx, pages_per_split=0, flags=0):
    out = torch.full(q.shape, float("nan"), dtype=torch.float32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = _lib.load().pkv_decode_noalloc(*_args(q, kc, vc, bt, ctx, out, pages_per_split, flags),
                                        status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_detail()
    assert int(status.item()) == 0
    return out


@pytest.mark.parametrize("force_generic", [False, True])
def test_no_alloc_matches_workspace_entry_point_on_two_calls(force_generic):
    flags = _lib.DECODE_FORCE_GENERIC if force_generic else 0
    # two different decodes in a row; both split long contexts, so the scratch
    # holds split-K partials and the second call overwrites the first's
    first = _case(1, 6, 12, 2, 128, 16, [3000, 1, 17, 512, 4096, 2049], torch.bfloat16)
    second = _case(2, 3, 28, 4, 128, 16, [700, 5000, 33], torch.bfloat16)
    for args in (first, second):
        ref = _with_workspace(*args, pages_per_split=8, flags=flags)
        got = _no_alloc(*args, pages_per_split=8, flags=flags)
        torch.cuda.synchronize()
        assert float((got - ref).abs().max()) <= ATOL["bfloat16"]


def test_no_alloc_fp32_small_case_twice():
    args = _case(3, 4, 12, 2, 128, 16, [37, 128, 300, 511], torch.float32)
    ref = _with_workspace(*args)
    for _ in range(2):
        got = _no_alloc(*args, pages_per_split=4)
        assert float((got - ref).abs().max()) <= ATOL["float32"]


def test_no_alloc_rejects_decodes_larger_than_its_scratch():
    q, kc, vc, bt, ctx = _case(4, 2, 12, 2, 128, 16, [40, 40], torch.bfloat16)
    out = torch.empty(q.shape, dtype=torch.float32, device=DEV)
    huge_batch, huge_blocks = 1 << 16, 1 << 14  # workspace far above the static scratch
    need = decode_workspace_bytes(huge_batch, 12, 2, 128, huge_blocks, 8)
    assert need > _lib.NOALLOC_SCRATCH_BYTES
    i64 = _lib.i64_array
    rc = _lib.load().pkv_decode_noalloc(
        q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), ctx.data_ptr(), out.data_ptr(),
        huge_batch, 12, 2, 128, 16, kc.shape[0], huge_blocks, i64(q.stride()), i64(kc.stride()),
        i64((huge_blocks, 1)), i64(out.stride()), _lib.DTYPE_BF16, _lib.DTYPE_BF16, 0.088, 8, 0, None,
        torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.ERR_WORKSPACE
    assert "static scratch" in _lib.last_detail()
