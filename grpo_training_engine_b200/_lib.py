"""ctypes binding of libpkv.so (the C ABI declared in include/pkv.h).

This is the only place that touches the shared library. It loads the in-tree
``libpkv.so`` (built by ``grpo_training_engine_b200.build``), declares every
entry point's argument types and turns negative status codes into Python
exceptions. A missing or unloadable library raises ``ImportError`` with the
reason — there is no fallback implementation.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libpkv.so"

ABI_VERSION = 10  # PKV_ABI_VERSION in include/pkv.h

SAMPLE_FORCE_RADIX = 1  # PKV_SAMPLE_FORCE_RADIX

DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_F16 = 2

OK = 0
ERR_INVALID_ARG = -1
ERR_UNSUPPORTED = -2
ERR_ALIGNMENT = -3
ERR_WORKSPACE = -4
ERR_CUDA = -5
ERR_TENSOR_MAP = -6

DEV_CTX_OUT_OF_RANGE = 1
DEV_PAGE_OUT_OF_RANGE = 2
DEV_WAIT_TIMEOUT = 4

DECODE_FORCE_GENERIC = 1
DECODE_EXACT_P = 2
DECODE_OUT_Q_DTYPE = 4  # PKV_DECODE_OUT_Q_DTYPE
DECODE_EARLY_START = 8  # PKV_DECODE_EARLY_START
DECODE_TEST_WAIT_TIMEOUT = 1 << 30  # PKV_DECODE_TEST_WAIT_TIMEOUT (tests of the bounded waits only)
LINEAR_NONE = 0  # PKV_LINEAR_NONE
LINEAR_SILU_GATE = 1  # PKV_LINEAR_SILU_GATE
LINEAR_WEIGHTS_STATIC = 0x100  # PKV_LINEAR_WEIGHTS_STATIC (flag OR'd into act)
NOALLOC_SCRATCH_BYTES = 32 << 20  # PKV_NOALLOC_SCRATCH_BYTES in include/pkv.h

_i32 = C.c_int32
_i64p = C.POINTER(C.c_int64)
_vp = C.c_void_p
_sz = C.c_size_t

# name -> (restype, argtypes); mirrors include/pkv.h one to one.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "pkv_abi_version": (C.c_int, []),
    "pkv_error_string": (C.c_char_p, [C.c_int]),
    "pkv_last_error_detail": (C.c_char_p, []),
    "pkv_append": (
        C.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i64p, _i64p, _i64p, _i32, _vp, _vp],
    ),
    "pkv_append_prompt": (
        C.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
         _i64p, _i64p, _i64p, _i32, _vp, _vp],
    ),
    "pkv_gather": (
        C.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i64p, _i64p, _i64p, _i32, _vp, _vp],
    ),
    "pkv_decode_pages_per_split": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32]),
    "pkv_decode_workspace_size": (_sz, [_i32, _i32, _i32, _i32, _i32, _i32]),
    "pkv_decode_plan": (C.c_int, [_vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _sz, _vp, _vp]),
    "pkv_decode_run": (
        C.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
         _i64p, _i64p, _i64p, _i64p, _i32, _i32, C.c_float, _i32, _i32, _vp, _sz, _vp, _vp],
    ),
    "pkv_append_decode_run": (
        C.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
         _i64p, _i64p, _i64p, _i64p, _i64p, _i32, _i32, C.c_float, _i32, _i32, _vp, _sz, _vp, _vp],
    ),
    "pkv_rope_append_decode_run": (
        C.c_int,
        [_vp, _vp, _vp, _vp, _vp, C.c_int64, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
         _i64p, _i64p, _i64p, _i64p, _i64p, _i32, _i32, C.c_float, _i32, _i32, _vp, _sz, _vp, _vp],
    ),
    "pkv_add_rmsnorm": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, C.c_int64, C.c_int64, C.c_int64,
                                  C.c_int64, C.c_float, _i32, _vp]),
    "pkv_silu_mul": (C.c_int, [_vp, _vp, _vp, _i32, _i32, C.c_int64, C.c_int64, _i32, _vp]),
    "pkv_rope_qk": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, C.c_int64, C.c_int64,
                              C.c_int64, C.c_int64, C.c_int64, _i32, _vp]),
    "pkv_sample_top_p": (C.c_int, [_vp, _i32, _i32, _i32, C.c_int64, C.c_float, C.c_float, _vp, _vp, _i32, _vp]),
    "pkv_decode": (
        C.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
         _i64p, _i64p, _i64p, _i64p, _i32, _i32, C.c_float, _i32, _i32, _vp, _sz, _vp, _vp],
    ),
    "pkv_decode_noalloc": (
        C.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
         _i64p, _i64p, _i64p, _i64p, _i32, _i32, C.c_float, _i32, _i32, _vp, _vp],
    ),
    "pkv_decode_kernel_kind": (C.c_int, [_vp, _i32, _i32, _i32, _i32, _i64p, _i32, _i32, _i32]),
    "pkv_linear": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, C.c_int64, C.c_int64, C.c_int64, _i32,
                             _i32, _vp, _vp]),
}


class PkvError(RuntimeError):
    """A libpkv entry point returned a negative status."""

    def __init__(self, fn: str, code: int, detail: str) -> None:
        self.code = code
        self.fn = fn
        super().__init__(f"{fn} failed: {error_string(code)} ({code}): {detail}")


_LIB: C.CDLL | None = None


def load() -> C.CDLL:
    """Load libpkv.so once; raise ImportError if it is absent or broken."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = Path(os.environ.get("PKV_LIBRARY", str(LIB_PATH)))
    if not path.exists():
        raise ImportError(
            f"{path} is missing: build it with `python grpo_training_engine_b200/build.py` "
            "(the paged-KV path has no non-CUDA implementation)"
        )
    try:
        lib = C.CDLL(str(path))
    except OSError as exc:  # pragma: no cover - depends on the environment
        raise ImportError(f"cannot load {path}: {exc}") from exc
    for name, (res, args) in SIGNATURES.items():
        try:
            fn = getattr(lib, name)
        except AttributeError as exc:
            raise ImportError(f"{path} is stale (no {name}): rebuild it with "
                              "`python grpo_training_engine_b200/build.py`") from exc
        fn.restype = res
        fn.argtypes = args
    if lib.pkv_abi_version() != ABI_VERSION:
        raise ImportError(f"{path} has ABI {lib.pkv_abi_version()}, this package needs {ABI_VERSION}: "
                          "rebuild it with `python grpo_training_engine_b200/build.py`")
    _LIB = lib
    return lib


def error_string(code: int) -> str:
    return load().pkv_error_string(code).decode()


def last_detail() -> str:
    return load().pkv_last_error_detail().decode()


def check(fn: str, code: int) -> int:
    if code < 0:
        raise PkvError(fn, code, last_detail())
    return code


def i64_array(values) -> C.Array:
    vals = [int(v) for v in values]
    return (C.c_int64 * len(vals))(*vals)


def ptr(t) -> int | None:
    """Device pointer of a tensor (None for None)."""
    return None if t is None else t.data_ptr()
