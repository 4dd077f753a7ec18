"""pkv_decode_noalloc: the decode entry point that allocates nothing.

Some callers cannot allocate device memory themselves — an FFI host that only
hands the library the tensors it owns, or a process whose GPU memory is held by
another framework's allocator. For them pkv_decode_noalloc takes no workspace
and uses a fixed scratch array built into libpkv.so instead. These tests call
it through the C ABI and check it against pkv_decode (with a workspace the test
allocates) on two calls in a row with different data, so a call that silently
reused the previous call's scratch contents would be caught. Both paths run the
same plan and kernels on the same inputs, so their outputs must be identical
bit for bit; the comparison with the CPU oracle uses the decode tolerance.

The scratch array has one device address per CUDA context. A host that makes
its own contexts with the driver API (cuCtxCreate) is one of the callers this
entry point serves, so one test runs it in a child process in a second context
next to the primary one. The file runs last so that a stop-at-first-failure
run has already run everything else.
"""

from __future__ import annotations

import ctypes as C
import math
import subprocess
import sys
import textwrap

import pytest
import torch

from conftest import ATOL, REPO
from grpo_training_engine_b200 import _lib, decode_workspace_bytes
from oracle import oracle

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
        assert torch.equal(got, ref)
        want = oracle.decode(*[t.cpu() for t in args])
        assert float((got.cpu() - want).abs().max()) <= ATOL["bfloat16"]


def test_no_alloc_fp32_small_case_twice():
    args = _case(3, 4, 12, 2, 128, 16, [37, 128, 300, 511], torch.float32)
    ref = _with_workspace(*args, pages_per_split=4)
    want = oracle.decode(*[t.cpu() for t in args])
    for _ in range(2):
        got = _no_alloc(*args, pages_per_split=4)
        assert torch.equal(got, ref)
        assert float((got.cpu() - want).abs().max()) <= ATOL["float32"]


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


# Child process: a driver-API host. It owns two contexts on GPU 0 (the primary
# one and one made with cuCtxCreate), allocates every buffer with cuMemAlloc in
# the context that uses it, and calls pkv_decode (workspace from cuMemAlloc) and
# pkv_decode_noalloc in each context, then in the primary context again. The
# no-alloc output must equal pkv_decode's bit for bit every time.
_CHILD = textwrap.dedent("""
    import ctypes as C, math, sys
    import numpy as np
    import torch
    sys.path.insert(0, sys.argv[1])
    from grpo_training_engine_b200 import _lib

    cu = C.CDLL("libcuda.so.1")
    vp, u64, sz, pp = C.c_void_p, C.c_uint64, C.c_size_t, C.POINTER(C.c_void_p)
    for name, args in {
        "cuInit": [C.c_uint], "cuDeviceGet": [C.POINTER(C.c_int), C.c_int],
        "cuDevicePrimaryCtxRetain": [pp, C.c_int], "cuDevicePrimaryCtxRelease_v2": [C.c_int],
        "cuCtxSetCurrent": [vp], "cuCtxCreate_v2": [pp, C.c_uint, C.c_int], "cuCtxDestroy_v2": [vp],
        "cuCtxSynchronize": [], "cuMemAlloc_v2": [C.POINTER(u64), sz], "cuMemFree_v2": [u64],
        "cuMemsetD8_v2": [u64, C.c_ubyte, sz], "cuMemcpyHtoD_v2": [u64, vp, sz],
        "cuMemcpyDtoH_v2": [vp, u64, sz],
    }.items():
        getattr(cu, name).argtypes = args
        getattr(cu, name).restype = C.c_int
    def ck(rc, what):
        if rc != 0:
            raise SystemExit(f"{what} failed: CUresult {rc}")
    ck(cu.cuInit(0), "cuInit")
    dev = C.c_int()
    ck(cu.cuDeviceGet(C.byref(dev), 0), "cuDeviceGet")
    primary = C.c_void_p()
    ck(cu.cuDevicePrimaryCtxRetain(C.byref(primary), dev), "cuDevicePrimaryCtxRetain")
    lib = _lib.load()

    def run_case(seed):
        g = torch.Generator().manual_seed(seed)
        B, hq, hkv, d, bs, pps = 5, 12, 2, 128, 16, 8
        ctxs = [900, 1, 33, 2000, 257]
        mb = max(math.ceil(c / bs) for c in ctxs) + 1
        nb = B * mb + 2
        host = {
            "q": torch.randn(B, hq, d, generator=g).to(torch.bfloat16),
            "k": torch.randn(nb, hkv, bs, d, generator=g).to(torch.bfloat16),
            "v": torch.randn(nb, hkv, bs, d, generator=g).to(torch.bfloat16),
            "bt": torch.randperm(nb, generator=g)[: B * mb].reshape(B, mb).int(),
            "ctx": torch.tensor(ctxs, dtype=torch.int32),
        }
        bufs = []
        def upload(t):
            raw = t.contiguous().view(torch.uint8).numpy() if t.dtype == torch.bfloat16 else t.contiguous().numpy()
            p = u64()
            ck(cu.cuMemAlloc_v2(C.byref(p), raw.nbytes), "cuMemAlloc")
            ck(cu.cuMemcpyHtoD_v2(p, raw.ctypes.data, raw.nbytes), "cuMemcpyHtoD")
            bufs.append(p)
            return p.value
        def alloc(n):
            p = u64()
            ck(cu.cuMemAlloc_v2(C.byref(p), n), "cuMemAlloc")
            ck(cu.cuMemsetD8_v2(p, 0, n), "cuMemsetD8")
            bufs.append(p)
            return p.value
        d_ = {k: upload(v) for k, v in host.items()}
        outs = [alloc(B * hq * d * 4) for _ in range(2)]
        status = alloc(4)
        ws_bytes = lib.pkv_decode_workspace_size(B, hq, hkv, d, mb, pps)
        ws = alloc(ws_bytes)
        i64 = _lib.i64_array
        common = [d_["q"], d_["k"], d_["v"], d_["bt"], d_["ctx"]]
        tail = [B, hq, hkv, d, bs, nb, mb, i64(host["q"].stride()), i64(host["k"].stride()),
                i64(host["bt"].stride()), i64((hq * d, d, 1)), _lib.DTYPE_BF16, _lib.DTYPE_BF16,
                1.0 / math.sqrt(d), pps, 0]
        rc = lib.pkv_decode(*common, outs[0], *tail, ws, ws_bytes, status, None)
        assert rc == 0, _lib.last_detail()
        rc = lib.pkv_decode_noalloc(*common, outs[1], *tail, status, None)
        assert rc == 0, _lib.last_detail()
        ck(cu.cuCtxSynchronize(), "cuCtxSynchronize")
        got = [np.empty(B * hq * d, dtype=np.float32) for _ in range(2)]
        for h, p in zip(got, outs):
            ck(cu.cuMemcpyDtoH_v2(h.ctypes.data, p, h.nbytes), "cuMemcpyDtoH")
        st = np.zeros(1, dtype=np.int32)
        ck(cu.cuMemcpyDtoH_v2(st.ctypes.data, status, 4), "cuMemcpyDtoH")
        for p in bufs:
            ck(cu.cuMemFree_v2(p), "cuMemFree")
        assert int(st[0]) == 0, f"status {int(st[0])}"
        assert np.isfinite(got[0]).all()
        assert np.array_equal(got[0], got[1]), "no-alloc output differs from pkv_decode"

    ck(cu.cuCtxSetCurrent(primary), "cuCtxSetCurrent(primary)")
    run_case(1)
    second = C.c_void_p()
    ck(cu.cuCtxCreate_v2(C.byref(second), 0, dev), "cuCtxCreate")
    run_case(2)  # current: the second context
    run_case(3)
    ck(cu.cuCtxSetCurrent(primary), "cuCtxSetCurrent(primary)")
    run_case(4)
    ck(cu.cuCtxDestroy_v2(second), "cuCtxDestroy")
    ck(cu.cuDevicePrimaryCtxRelease_v2(dev), "cuDevicePrimaryCtxRelease")
    print("contexts ok")
""")


def test_no_alloc_in_a_second_driver_api_context():
    res = subprocess.run([sys.executable, "-c", _CHILD, str(REPO)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    assert "contexts ok" in res.stdout
