"""The C ABI: libpkv.so loads, exports exactly what include/pkv.h declares, and
its host-side argument checks work without a GPU (no kernel is launched)."""

from __future__ import annotations

import ctypes as C
import re
import subprocess

import pytest

from conftest import REPO
from grpo_training_engine_b200 import _lib

HEADER = REPO / "include" / "pkv.h"


def _declared() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"\b(pkv_[a-z0-9_]+)\s*\(", text))


def test_library_loads():
    lib = _lib.load()
    assert lib.pkv_abi_version() == _lib.ABI_VERSION == 10


def test_every_declared_symbol_is_exported():
    lib = _lib.load()
    names = _declared()
    assert {"pkv_append", "pkv_decode", "pkv_gather", "pkv_append_prompt"} <= names
    for name in names:
        assert hasattr(lib, name), name
    assert names == set(_lib.SIGNATURES), "ctypes signatures must cover the header exactly"


def test_only_pkv_symbols_are_exported():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    syms = {line.split()[-1] for line in out.splitlines() if line.strip()}
    assert syms and all(s.startswith("pkv_") for s in syms), sorted(s for s in syms if not s.startswith("pkv_"))


def test_error_strings():
    for code in range(-6, 1):
        assert _lib.error_string(code) not in ("", "unknown status")
    assert _lib.error_string(-99) == "unknown status"


def _strides(*vals):
    return _lib.i64_array(vals)


def test_append_rejects_bad_sizes_without_launching():
    lib = _lib.load()
    rc = lib.pkv_append(None, None, None, None, None, None, 2, 0, 128, 16, 10, 4,
                        _strides(256, 128, 1), _strides(4096, 2048, 128, 1), _strides(4, 1), 1, None, None)
    assert rc == _lib.ERR_INVALID_ARG
    assert "heads=0" in _lib.last_detail()
    rc = lib.pkv_append(None, None, None, None, None, None, 2, 2, 128, 16, 10, 4,
                        _strides(256, 128, 1), _strides(4096, 2048, 128, 1), _strides(4, 1), 9, None, None)
    assert rc == _lib.ERR_UNSUPPORTED
    # zero batch is a no-op, even with NULL pointers
    rc = lib.pkv_append(None, None, None, None, None, None, 0, 2, 128, 16, 10, 4,
                        _strides(256, 128, 1), _strides(4096, 2048, 128, 1), _strides(4, 1), 1, None, None)
    assert rc == _lib.OK


def test_decode_checks_and_workspace_query():
    lib = _lib.load()
    ws = lib.pkv_decode_workspace_size(1024, 12, 2, 128, 513, 64)
    assert ws > 1024 * 2 * 6 * 128 * 4
    assert lib.pkv_decode_workspace_size(4, 12, 5, 128, 32, 0) == 0  # 12 % 5 != 0
    assert lib.pkv_decode_pages_per_split(4, 12, 2, 128, 32, 16) == 16
    p = lib.pkv_decode_pages_per_split(1024, 12, 2, 128, 513, 0)
    assert 8 <= p <= 512 and p % 8 == 0

    # plan without a workspace is refused before any launch
    rc = lib.pkv_decode_plan(None, 4, 12, 2, 128, 16, 32, 0, None, 0, None, None)
    assert rc == _lib.ERR_WORKSPACE
    rc = lib.pkv_decode(None, None, None, None, None, None, 4, 12, 5, 128, 16, 10, 4,
                        _strides(1, 1, 1), _strides(1, 1, 1, 1), _strides(1, 1), _strides(1, 1, 1),
                        1, 1, 0.1, 0, 0, None, 0, None, None)
    assert rc == _lib.ERR_INVALID_ARG
    assert "multiple" in _lib.last_detail()


def test_default_split_length_cost_model():
    """Without a GPU the library assumes a B200's 148 SMs."""
    pps = _lib.load().pkv_decode_pages_per_split
    assert pps(128, 12, 2, 128, 64, 0) == 64      # config 3: 256 whole sequences fill 148 SMs, no split
    assert pps(1024, 12, 2, 128, 512, 0) == 512   # config 4: every sequence one unit, no merge
    assert pps(64, 28, 4, 128, 2048, 0) == 512    # config 5: the longest splits
    p = pps(4, 12, 2, 128, 2048, 0)               # 8 long sequences: split to fill the SMs once
    assert 8 * -(-2048 // p) <= 148 and 8 * -(-2048 // (p + 8)) < 148 <= 8 * -(-2048 // (p - 8))
    # a few short sequences leave most SMs idle: split them (the tensor-core
    # kernel merges inside the launch, so a split costs no extra launch)
    assert pps(4, 12, 2, 128, 33, 0) < 33


def test_kernel_kind_selection():
    lib = _lib.load()
    aligned = C.c_void_p(1 << 20)
    cs = _strides(2 * 16 * 128, 16 * 128, 128, 1)
    tc = lib.pkv_decode_kernel_kind(aligned, 12, 2, 128, 16, cs, 1, 1, 0)
    assert tc == 1
    assert lib.pkv_decode_kernel_kind(aligned, 12, 2, 128, 16, cs, 1, 1, _lib.DECODE_FORCE_GENERIC) == 0
    assert lib.pkv_decode_kernel_kind(aligned, 12, 2, 128, 16, cs, 0, 0, 0) == 0  # fp32 -> CUDA cores
    assert lib.pkv_decode_kernel_kind(aligned, 2, 2, 8, 4, _strides(64, 32, 8, 1), 1, 1, 0) == 0  # tiny
    assert lib.pkv_decode_kernel_kind(C.c_void_p((1 << 20) + 2), 12, 2, 128, 16, cs, 1, 1, 0) == 0


def test_ops_reject_cpu_tensors_with_reference_message():
    import torch

    from grpo_training_engine_b200 import paged_attention_decode, paged_kv_append

    kc = torch.zeros(4, 2, 16, 8, dtype=torch.bfloat16)
    bt = torch.zeros(1, 2, dtype=torch.int32)
    ctx = torch.zeros(1, dtype=torch.int32)
    with pytest.raises(ValueError, match="inputs and caches must be on CUDA device."):
        paged_kv_append(torch.zeros(1, 2, 8, dtype=torch.bfloat16), torch.zeros(1, 2, 8, dtype=torch.bfloat16),
                        kc, kc.clone(), bt, ctx)
    with pytest.raises(ValueError, match="inputs and caches must be on CUDA device."):
        paged_attention_decode(torch.zeros(1, 4, 8, dtype=torch.bfloat16), kc, kc.clone(), bt, ctx)
    with pytest.raises(ValueError, match="must be divisible"):
        paged_attention_decode(torch.zeros(1, 3, 8, dtype=torch.bfloat16), kc, kc.clone(), bt, ctx)


def test_linear_host_checks_without_a_gpu():
    """pkv_linear refuses what it cannot serve before touching the GPU; a call
    that passes every check stops at the tensor-map encoder here (no driver)."""
    lib = _lib.load()
    A = C.c_void_p(1 << 20)  # 16-byte aligned fake device addresses (never dereferenced)
    B = C.c_void_p(1 << 21)
    O = C.c_void_p(1 << 22)
    bf16, none, silu, static = _lib.DTYPE_BF16, _lib.LINEAR_NONE, _lib.LINEAR_SILU_GATE, _lib.LINEAR_WEIGHTS_STATIC

    def call(x=A, w=B, w_up=None, bias=None, out=O, rows=128, n=1536, k=1536, xs=1536, ws=1536, os_=1536,
             dtype=bf16, act=none):
        return lib.pkv_linear(x, w, w_up, bias, out, rows, n, k, xs, ws, os_, dtype, act, None, None)

    assert call(rows=0) == _lib.ERR_INVALID_ARG
    assert call(rows=129) == _lib.ERR_INVALID_ARG
    assert call(n=0) == _lib.ERR_INVALID_ARG
    assert call(dtype=_lib.DTYPE_F32) == _lib.ERR_UNSUPPORTED
    assert call(act=2) == _lib.ERR_INVALID_ARG
    assert call(act=static | 2) == _lib.ERR_INVALID_ARG
    assert call(k=100, xs=100, ws=100) == _lib.ERR_UNSUPPORTED          # K not a multiple of 64
    assert call(act=silu, n=1000, os_=1000) == _lib.ERR_UNSUPPORTED     # the gate needs n % 64 == 0
    assert call(act=silu, bias=A) == _lib.ERR_UNSUPPORTED               # and no bias
    assert call(w_up=A) == _lib.ERR_INVALID_ARG                         # w_up only with the gate
    assert call(x=None) == _lib.ERR_INVALID_ARG
    assert call(x=C.c_void_p((1 << 20) + 2)) == _lib.ERR_ALIGNMENT
    assert call(xs=1000) == _lib.ERR_ALIGNMENT                          # row stride < k
    assert call(os_=1537) == _lib.ERR_ALIGNMENT                         # out rows not 16-byte multiples
    assert "pkv_linear" in _lib.last_detail()
    # every check passes (the static-weights flag, the gate with separate up rows): only the
    # tensor-map encoder, which needs the driver, is left
    for act, w_up in ((none, None), (static, None), (silu | static, A), (silu, None)):
        assert call(act=act, w_up=w_up) == _lib.ERR_TENSOR_MAP, act
