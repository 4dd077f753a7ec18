"""Kernel-level paged-KV operations on torch tensors, calling libpkv.so.

Each function validates its tensors, passes raw device pointers, element
strides and the current CUDA stream through the C ABI (include/pkv.h) and
returns without synchronising. There is no non-CUDA implementation: CPU
tensors are rejected with the reference's ValueError, and a missing
libpkv.so raises ImportError.

Reference correspondence (src/triton_kernels/paged_kv.py):
  paged_kv_append        _paged_kv_update_kernel launch   :253-319, :730-752
  paged_attention_decode _paged_attention_decode_kernel   :63-251,  :754-783
  paged_kv_append_prompt _prefill_paged_cache scatter     :572-586
  gather_kv              the kernel's block-table addressing written densely :98-131
"""

from __future__ import annotations

import contextlib
import functools
import math
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib


@functools.lru_cache(maxsize=512)
def _strides(values: tuple) -> object:
    """ctypes int64 array of a stride tuple, built once per distinct tuple (the
    library only reads it; the arrays are kept alive by the cache)."""
    return _lib.i64_array(values)


_NULL_CTX = contextlib.nullcontext()


def _device_ctx(dev: torch.device):
    """torch.cuda.device(dev) only when dev is not already the current device."""
    return _NULL_CTX if dev.index == torch.cuda.current_device() else torch.cuda.device(dev)

_DTYPES = {
    torch.float32: _lib.DTYPE_F32,
    torch.bfloat16: _lib.DTYPE_BF16,
    torch.float16: _lib.DTYPE_F16,
}


def _dtype_code(t: torch.Tensor, what: str) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise ValueError(f"{what} must be float32, bfloat16 or float16, got {t.dtype}.") from None


def _require_cuda(*tensors: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("inputs and caches must be on CUDA device.")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"all tensors must be on one device, got {dev} and {t.device}.")
    assert dev is not None
    return dev


def _as_i32(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.int32 else t.to(torch.int32)


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _check_cache_pair(k_cache: torch.Tensor, v_cache: torch.Tensor) -> None:
    if k_cache.ndim != 4 or v_cache.ndim != 4:
        raise ValueError("k_cache/v_cache must be [num_blocks, heads, block, head_dim].")
    if k_cache.shape != v_cache.shape:
        raise ValueError("k_cache and v_cache must have identical shapes.")
    if k_cache.dtype != v_cache.dtype:
        raise ValueError("k_cache and v_cache must have the same dtype.")
    if k_cache.stride() != v_cache.stride():
        raise ValueError("k_cache and v_cache must have identical strides.")


def _check_tables(block_tables: torch.Tensor, context_lens: torch.Tensor, batch: int) -> None:
    if block_tables.ndim != 2:
        raise ValueError(f"block_tables must be [batch, max_blocks], got {tuple(block_tables.shape)}.")
    if context_lens.ndim != 1:
        raise ValueError(f"context_lens must be [batch], got {tuple(context_lens.shape)}.")
    if block_tables.shape[0] != batch:
        raise ValueError("block_tables batch dimension must match input_ids batch.")
    if context_lens.shape[0] != batch:
        raise ValueError("context_lens batch dimension must match input_ids batch.")


def _status_ptr(status: Optional[torch.Tensor]) -> Optional[int]:
    if status is None:
        return None
    if status.dtype != torch.int32 or status.numel() < 1 or not status.is_cuda:
        raise ValueError("status must be a CUDA int32 tensor with at least one element.")
    return status.data_ptr()


# ---------------------------------------------------------------------------
# append / prompt append / gather
# ---------------------------------------------------------------------------
def paged_kv_append(
    k_new: torch.Tensor,
    v_new: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    *,
    status: Optional[torch.Tensor] = None,
) -> None:
    """Write k_new/v_new [B, H, D] at position context_lens[b] (pre-append) in place.

    Same slot rule as the reference update kernel (paged_kv.py:277-284); the
    payload is copied bit for bit.
    """
    _check_cache_pair(k_cache, v_cache)
    if k_new.ndim != 3 or k_new.shape != v_new.shape:
        raise ValueError("k_new/v_new must be matching [batch, heads, head_dim] tensors.")
    if k_new.stride() != v_new.stride():
        raise ValueError("k_new and v_new must have identical strides.")
    batch, heads, head_dim = k_new.shape
    num_blocks, cache_heads, block_size, cache_dim = k_cache.shape
    if heads != cache_heads or head_dim != cache_dim:
        raise ValueError(
            f"k_new {tuple(k_new.shape)} does not match cache heads/head_dim ({cache_heads}, {cache_dim})."
        )
    if k_new.dtype != k_cache.dtype or v_new.dtype != k_cache.dtype:
        raise ValueError("k_new/v_new must have the cache dtype.")
    _check_tables(block_tables, context_lens, batch)
    dev = _require_cuda(k_new, v_new, k_cache, v_cache, block_tables, context_lens, status)
    bt = _as_i32(block_tables)
    ctx = _as_i32(context_lens)
    lib = _lib.load()
    with _device_ctx(dev):
        _lib.check(
            "pkv_append",
            lib.pkv_append(
                k_new.data_ptr(), v_new.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                bt.data_ptr(), ctx.data_ptr(), batch, heads, head_dim, block_size, num_blocks,
                bt.shape[1], _strides(k_new.stride()), _strides(k_cache.stride()),
                _strides(bt.stride()), _dtype_code(k_cache, "k_cache"), _status_ptr(status),
                _stream(dev),
            ),
        )


def paged_kv_append_prompt(
    k: torch.Tensor,
    v: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    start_pos: Optional[torch.Tensor] = None,
    lens: Optional[torch.Tensor] = None,
    *,
    status: Optional[torch.Tensor] = None,
) -> None:
    """Bulk prompt write: k/v [B, H, T, D] (HF past_key_values layout) into pages.

    Position start_pos[b] + t for t < lens[b] (defaults 0 and T), the
    addressing of the reference prefill scatter (paged_kv.py:576-586) done
    in one launch instead of B x T x L slice assignments.
    """
    _check_cache_pair(k_cache, v_cache)
    if k.ndim != 4 or k.shape != v.shape or k.stride() != v.stride():
        raise ValueError("k/v must be matching [batch, heads, seq_len, head_dim] tensors.")
    batch, heads, seq_len, head_dim = k.shape
    num_blocks, cache_heads, block_size, cache_dim = k_cache.shape
    if heads != cache_heads or head_dim != cache_dim:
        raise ValueError(f"k {tuple(k.shape)} does not match cache heads/head_dim ({cache_heads}, {cache_dim}).")
    if k.dtype != k_cache.dtype or v.dtype != k_cache.dtype:
        raise ValueError("k/v must have the cache dtype.")
    if block_tables.ndim != 2 or block_tables.shape[0] != batch:
        raise ValueError("block_tables must be [batch, max_blocks].")
    for name, t in (("start_pos", start_pos), ("lens", lens)):
        if t is not None and (t.ndim != 1 or t.shape[0] != batch):
            raise ValueError(f"{name} must be [batch].")
    dev = _require_cuda(k, v, k_cache, v_cache, block_tables, start_pos, lens, status)
    bt = _as_i32(block_tables)
    sp = None if start_pos is None else _as_i32(start_pos)
    ln = None if lens is None else _as_i32(lens)
    lib = _lib.load()
    with _device_ctx(dev):
        _lib.check(
            "pkv_append_prompt",
            lib.pkv_append_prompt(
                k.data_ptr(), v.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), bt.data_ptr(),
                _lib.ptr(sp), _lib.ptr(ln), batch, heads, seq_len, head_dim, block_size, num_blocks,
                bt.shape[1], _strides(k.stride()), _strides(k_cache.stride()),
                _strides(bt.stride()), _dtype_code(k_cache, "k_cache"), _status_ptr(status),
                _stream(dev),
            ),
        )


def gather_kv(
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    max_tokens: Optional[int] = None,
    *,
    status: Optional[torch.Tensor] = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Dense K, V [B, H, T, D] of the paged cache; positions >= context_lens[b] are zero.

    max_tokens defaults to the block-table capacity max_blocks * block_size.
    """
    _check_cache_pair(k_cache, v_cache)
    batch = block_tables.shape[0] if block_tables.ndim == 2 else -1
    _check_tables(block_tables, context_lens, batch)
    dev = _require_cuda(k_cache, v_cache, block_tables, context_lens, status)
    num_blocks, heads, block_size, head_dim = k_cache.shape
    bt = _as_i32(block_tables)
    ctx = _as_i32(context_lens)
    if max_tokens is None:
        max_tokens = bt.shape[1] * block_size
    k_out = torch.empty((batch, heads, max_tokens, head_dim), dtype=k_cache.dtype, device=dev)
    v_out = torch.empty_like(k_out)
    lib = _lib.load()
    with _device_ctx(dev):
        _lib.check(
            "pkv_gather",
            lib.pkv_gather(
                k_cache.data_ptr(), v_cache.data_ptr(), bt.data_ptr(), ctx.data_ptr(),
                k_out.data_ptr(), v_out.data_ptr(), batch, heads, head_dim, block_size, num_blocks,
                bt.shape[1], max_tokens, _strides(k_cache.stride()),
                _strides(bt.stride()), _strides(k_out.stride()),
                _dtype_code(k_cache, "k_cache"), _status_ptr(status), _stream(dev),
            ),
        )
    return k_out, v_out


# ---------------------------------------------------------------------------
# decode attention
# ---------------------------------------------------------------------------
@dataclass
class DecodePlan:
    """A decode work plan in a device workspace, valid for one context_lens.

    A plan depends only on context_lens and the sizes, so a caller that runs
    several layers with the same context_lens (one decode step of a model)
    makes one plan and calls ``paged_attention_decode(..., plan=plan)`` per
    layer. The workspace is also the split-K scratch of every call that uses
    the plan: calls sharing a plan must be ordered on one stream.
    ``pages_per_split`` is the split-length argument every call of the plan
    passes (0: the library's heuristic); ``chosen_pages_per_split()`` reads the
    length the plan kernel used back from the workspace (a device sync).
    """

    batch: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    max_blocks: int
    pages_per_split: int
    workspace: torch.Tensor
    context_lens: torch.Tensor

    def chosen_pages_per_split(self) -> int:
        """The split length the plan kernel wrote into the workspace header."""
        return int(self.workspace[:8].view(torch.int32)[1].item())

    def matches(self, batch, num_q_heads, num_kv_heads, head_dim, block_size, max_blocks) -> bool:
        return (self.batch, self.num_q_heads, self.num_kv_heads, self.head_dim, self.block_size, self.max_blocks) == (
            batch, num_q_heads, num_kv_heads, head_dim, block_size, max_blocks)


def decode_workspace_bytes(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, pages_per_split=0) -> int:
    n = _lib.load().pkv_decode_workspace_size(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, pages_per_split)
    if n == 0:
        raise ValueError("invalid decode geometry for the workspace size query.")
    return int(n)


def _pages_per_split(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, num_splits, pages_per_split) -> int:
    """The split-length argument of the C ABI: pages_per_split, or the length
    that caps the splits per sequence at num_splits, or 0 (the library's
    heuristic, which lets the plan kernel pick the length from the actual
    context lengths when the batch has fewer units than SMs)."""
    if pages_per_split <= 0 and num_splits and num_splits > 0:
        pages_per_split = max(1, math.ceil(max(max_blocks, 1) / num_splits))
    pages_per_split = max(0, int(pages_per_split))
    _lib.check(
        "pkv_decode_pages_per_split",
        _lib.load().pkv_decode_pages_per_split(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, pages_per_split),
    )
    return pages_per_split


def plan_decode(
    context_lens: torch.Tensor,
    num_q_heads: int,
    num_kv_heads: int,
    head_dim: int,
    block_size: int,
    max_blocks: int,
    num_splits: int = 0,
    *,
    pages_per_split: int = 0,
    workspace: Optional[torch.Tensor] = None,
    status: Optional[torch.Tensor] = None,
) -> DecodePlan:
    """Plan the split-K decode of all sequences for one context_lens (post-append lengths)."""
    if context_lens.ndim != 1:
        raise ValueError(f"context_lens must be [batch], got {tuple(context_lens.shape)}.")
    if num_q_heads % num_kv_heads != 0:
        raise ValueError(f"num_heads ({num_q_heads}) must be divisible by num_kv_heads ({num_kv_heads}).")
    dev = _require_cuda(context_lens, workspace, status)
    batch = context_lens.shape[0]
    ctx = _as_i32(context_lens)
    pps = _pages_per_split(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, num_splits, pages_per_split)
    need = decode_workspace_bytes(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, pps)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
    lib = _lib.load()
    with _device_ctx(dev):
        _lib.check(
            "pkv_decode_plan",
            lib.pkv_decode_plan(
                ctx.data_ptr(), batch, num_q_heads, num_kv_heads, head_dim, block_size, max_blocks, pps,
                workspace.data_ptr(), workspace.numel() * workspace.element_size(), _status_ptr(status),
                _stream(dev),
            ),
        )
    return DecodePlan(batch, num_q_heads, num_kv_heads, head_dim, block_size, max_blocks, pps, workspace, ctx)


def paged_attention_decode(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    scale: Optional[float] = None,
    out: Optional[torch.Tensor] = None,
    num_splits: int = 0,
    *,
    pages_per_split: int = 0,
    plan: Optional[DecodePlan] = None,
    force_generic: bool = False,
    exact: bool = False,
    status: Optional[torch.Tensor] = None,
    k_new: Optional[torch.Tensor] = None,
    v_new: Optional[torch.Tensor] = None,
    out_dtype: Optional[torch.dtype] = None,
    rope: Optional[tuple[torch.Tensor, torch.Tensor]] = None,
    early_start: bool = False,
) -> torch.Tensor:
    """Single-query attention over the paged cache; returns fp32 [B, Hq, D].

    q is [B, Hq, D]; the caches are [num_blocks, Hkv, block_size, D] with
    Hq a multiple of Hkv (query head h reads cache head h // (Hq // Hkv),
    the grouped-query mapping of HF repeat_kv). Hq == Hkv is the reference's
    head-replicated layout. context_lens are POST-append lengths
    (paged_kv.py:697,761,938); scale defaults to 1/sqrt(D) (paged_kv.py:681,900).
    num_splits > 0 caps the number of split-K chunks per sequence;
    pages_per_split > 0 sets the chunk length directly; both 0 = heuristic.
    The tensor-core kernel multiplies the softmax weights by V in 16 bits
    (max-abs error a few 1e-3 for N(0,1) data); exact=True keeps ~17
    significant bits of the weights at some speed cost. The CUDA-core kernel
    (fp32 caches, force_generic=True) is fp32 throughout.

    With k_new / v_new ([B, Hkv, D], cache dtype) the call is one decode step
    of a layer including the append: the new token is written at position
    context_lens[b] - 1 (context_lens stay POST-append) and attended to, in
    a single launch on the tensor-core kernel (C ABI pkv_append_decode_run).
    It writes the cache bytes paged_kv_append(..., context_lens - 1) writes.

    With rope=(cos, sin) ([B, D], q's dtype) and k_new / v_new, q and k_new
    are the rows before RoPE and the launch rotates them as rope_qk does (C ABI
    pkv_rope_append_decode_run; tensor-core kernel only, PkvError otherwise).

    out_dtype=q.dtype (bf16 / fp16 q) returns the output in q's dtype, each
    fp32 result rounded to nearest: the values of ``.to(q.dtype)`` of the fp32
    output, without a separate conversion launch.

    early_start=True promises that the previous kernel queued on the stream
    wrote none of the plan, the block tables, the context lengths and the
    caches, and that the kernels before it are complete once it lets this
    launch start: true for every layer's decode launch of a step after the
    first (each follows an earlier decode launch, which lets the next launch
    start only after its own wait), not for the first (behind the plan) nor
    one behind a separate append. The tensor-core launch then schedules its
    first unit and starts loading its pages before that kernel has finished;
    q, the new rows and cos / sin are still read after it. Results are
    unchanged.
    """
    _check_cache_pair(k_cache, v_cache)
    if q.ndim != 3:
        raise ValueError(f"q must be [batch, heads, head_dim], got {tuple(q.shape)}.")
    batch, hq, head_dim = q.shape
    num_blocks, hkv, block_size, cache_dim = k_cache.shape
    if cache_dim != head_dim:
        raise ValueError(f"q head_dim {head_dim} does not match cache head_dim {cache_dim}.")
    if hq % hkv != 0:
        raise ValueError(f"num_heads ({hq}) must be divisible by num_kv_heads ({hkv}).")
    _check_tables(block_tables, context_lens, batch)
    dev = _require_cuda(q, k_cache, v_cache, block_tables, context_lens, out, status)
    if out_dtype is None:
        out_dtype = out.dtype if out is not None else torch.float32
    if out_dtype not in (torch.float32, q.dtype):
        raise ValueError(f"out_dtype must be float32 or q's dtype ({q.dtype}), got {out_dtype}.")
    if out is None:
        out = torch.empty((batch, hq, head_dim), dtype=out_dtype, device=dev)
    elif out.dtype != out_dtype or tuple(out.shape) != (batch, hq, head_dim):
        raise ValueError(f"out must be a {out_dtype} [batch, heads, head_dim] tensor.")
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    bt = _as_i32(block_tables)
    max_blocks = bt.shape[1]
    if plan is None:
        plan = plan_decode(context_lens, hq, hkv, head_dim, block_size, max_blocks, num_splits,
                           pages_per_split=pages_per_split, status=status)
    elif not plan.matches(batch, hq, hkv, head_dim, block_size, max_blocks):
        raise ValueError("decode plan was made for a different geometry.")
    lib = _lib.load()
    ws = plan.workspace
    if rope is not None and k_new is None:
        raise ValueError("rope needs k_new / v_new (RoPE runs with the fused append).")
    flags = (_lib.DECODE_FORCE_GENERIC if force_generic else 0) | (_lib.DECODE_EXACT_P if exact else 0)
    if early_start:
        flags |= _lib.DECODE_EARLY_START
    if out.dtype != torch.float32:
        flags |= _lib.DECODE_OUT_Q_DTYPE
    if k_new is not None or v_new is not None:
        if k_new is None or v_new is None:
            raise ValueError("k_new and v_new must be given together.")
        if k_new.ndim != 3 or k_new.shape != v_new.shape or tuple(k_new.shape) != (batch, hkv, head_dim):
            raise ValueError(f"k_new/v_new must be matching [batch, num_kv_heads, head_dim] = "
                             f"{(batch, hkv, head_dim)} tensors.")
        if k_new.stride() != v_new.stride():
            raise ValueError("k_new and v_new must have identical strides.")
        if k_new.dtype != k_cache.dtype or v_new.dtype != k_cache.dtype:
            raise ValueError("k_new/v_new must have the cache dtype.")
        _require_cuda(k_new, v_new, k_cache)
        if rope is not None:
            cos, sin = rope
            if cos.shape != (batch, head_dim) or sin.shape != cos.shape or cos.stride() != sin.stride() \
                    or cos.stride(1) != 1 or cos.dtype != q.dtype or sin.dtype != q.dtype:
                raise ValueError("rope cos / sin must be matching [batch, head_dim] tensors of q's dtype "
                                 "with contiguous rows.")
            _require_cuda(cos, sin)
            with _device_ctx(dev):
                _lib.check(
                    "pkv_rope_append_decode_run",
                    lib.pkv_rope_append_decode_run(
                        q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                        cos.stride(0), k_cache.data_ptr(), v_cache.data_ptr(), bt.data_ptr(),
                        plan.context_lens.data_ptr(), out.data_ptr(), batch, hq, hkv, head_dim, block_size,
                        num_blocks, max_blocks, _strides(q.stride()), _strides(k_new.stride()),
                        _strides(k_cache.stride()), _strides(bt.stride()), _strides(out.stride()),
                        _dtype_code(q, "q"), _dtype_code(k_cache, "k_cache"), float(scale), plan.pages_per_split,
                        flags, ws.data_ptr(), ws.numel() * ws.element_size(), _status_ptr(status), _stream(dev),
                    ),
                )
            return out
        with _device_ctx(dev):
            _lib.check(
                "pkv_append_decode_run",
                lib.pkv_append_decode_run(
                    q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                    bt.data_ptr(), plan.context_lens.data_ptr(), out.data_ptr(), batch, hq, hkv, head_dim,
                    block_size, num_blocks, max_blocks, _strides(q.stride()), _strides(k_new.stride()),
                    _strides(k_cache.stride()), _strides(bt.stride()), _strides(out.stride()),
                    _dtype_code(q, "q"), _dtype_code(k_cache, "k_cache"), float(scale), plan.pages_per_split,
                    flags, ws.data_ptr(), ws.numel() * ws.element_size(), _status_ptr(status), _stream(dev),
                ),
            )
        return out
    with _device_ctx(dev):
        _lib.check(
            "pkv_decode_run",
            lib.pkv_decode_run(
                q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), bt.data_ptr(), plan.context_lens.data_ptr(),
                out.data_ptr(), batch, hq, hkv, head_dim, block_size, num_blocks, max_blocks,
                _strides(q.stride()), _strides(k_cache.stride()), _strides(bt.stride()),
                _strides(out.stride()), _dtype_code(q, "q"), _dtype_code(k_cache, "k_cache"),
                float(scale), plan.pages_per_split, flags, ws.data_ptr(), ws.numel() * ws.element_size(),
                _status_ptr(status), _stream(dev),
            ),
        )
    return out


# ---------------------------------------------------------------------------
# decode-step element-wise steps
# ---------------------------------------------------------------------------
def add_rmsnorm(
    x: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    residual: Optional[torch.Tensor] = None,
) -> tuple[torch.Tensor, Optional[torch.Tensor]]:
    """RMSNorm of x [rows, hidden] (after adding residual, if given) in one launch.

    Returns (normed, x + residual or None), with the rounding points of HF's
    Qwen2RMSNorm: the sum rounded to the dtype, fp32 statistics,
    dtype(s * rsqrt(mean(s^2) + eps)) scaled by weight (C ABI pkv_add_rmsnorm).
    """
    if x.ndim != 2 or x.stride(1) != 1:
        raise ValueError("x must be [rows, hidden] with contiguous rows.")
    rows, hidden = x.shape
    if weight.shape != (hidden,) or weight.dtype != x.dtype or not weight.is_contiguous():
        raise ValueError("weight must be a contiguous [hidden] tensor of x's dtype.")
    if residual is not None and (residual.shape != x.shape or residual.dtype != x.dtype or residual.stride(1) != 1):
        raise ValueError("residual must match x.")
    dev = _require_cuda(x, weight, residual)
    out = torch.empty_like(x, memory_format=torch.contiguous_format)
    total = torch.empty_like(out) if residual is not None else None
    with _device_ctx(dev):
        _lib.check(
            "pkv_add_rmsnorm",
            _lib.load().pkv_add_rmsnorm(
                x.data_ptr(), residual.data_ptr() if residual is not None else None, weight.data_ptr(),
                total.data_ptr() if total is not None else None, out.data_ptr(), rows, hidden, x.stride(0),
                residual.stride(0) if residual is not None else 0, hidden, hidden, float(eps),
                _dtype_code(x, "x"), _stream(dev)),
        )
    return out, total


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """dtype(dtype(silu(gate)) * up) for [rows, cols] tensors in one launch (C ABI pkv_silu_mul):
    the gated activation of a Qwen2 MLP with the rounding of F.silu(gate) * up."""
    if gate.ndim != 2 or gate.shape != up.shape or gate.dtype != up.dtype or gate.stride(1) != 1 or up.stride(1) != 1:
        raise ValueError("gate and up must be matching [rows, cols] tensors with contiguous rows.")
    dev = _require_cuda(gate, up)
    out = torch.empty(gate.shape, dtype=gate.dtype, device=dev)
    with _device_ctx(dev):
        _lib.check(
            "pkv_silu_mul",
            _lib.load().pkv_silu_mul(gate.data_ptr(), up.data_ptr(), out.data_ptr(), gate.shape[0], gate.shape[1],
                                     gate.stride(0), up.stride(0), _dtype_code(gate, "gate"), _stream(dev)),
        )
    return out


def rope_qk(
    q: torch.Tensor,
    k: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    num_q_heads: int,
    num_kv_heads: int,
    head_dim: int,
    k_out: Optional[torch.Tensor] = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """RoPE of one new query / key row per sequence, one launch.

    q [rows, Hq * D], k [rows, Hkv * D] (the projections' outputs), cos / sin
    [rows, D]; returns q [rows, Hq, D] (contiguous) and k [rows, Hkv, D] equal to
    HF's apply_rotary_pos_emb of the same rows (C ABI pkv_rope_qk). With k_out
    ([rows, Hkv * D], contiguous rows; k itself rotates k in place) the keys are
    written there and the returned k is its [rows, Hkv, D] view.
    """
    rows = q.shape[0]
    if (q.shape != (rows, num_q_heads * head_dim) or k.shape != (rows, num_kv_heads * head_dim)
            or q.stride(1) != 1 or k.stride(1) != 1):
        raise ValueError("q / k must be [rows, heads * head_dim] with contiguous rows.")
    if cos.shape != (rows, head_dim) or sin.shape != cos.shape or cos.stride() != sin.stride() or cos.stride(1) != 1:
        raise ValueError("cos / sin must be matching [rows, head_dim] tensors with contiguous rows.")
    if not (q.dtype == k.dtype == cos.dtype == sin.dtype):
        raise ValueError("q, k, cos and sin must share one dtype.")
    dev = _require_cuda(q, k, cos, sin)
    qo = torch.empty(rows, num_q_heads, head_dim, dtype=q.dtype, device=dev)
    if k_out is None:
        ko = torch.empty(rows, num_kv_heads, head_dim, dtype=k.dtype, device=dev)
        k_rows = num_kv_heads * head_dim
    else:
        if k_out.shape != k.shape or k_out.dtype != k.dtype or k_out.stride(1) != 1:
            raise ValueError("k_out must match k: [rows, heads * head_dim] with contiguous rows.")
        _require_cuda(k_out)
        ko, k_rows = k_out.view(rows, num_kv_heads, head_dim), k_out.stride(0)
    with _device_ctx(dev):
        _lib.check(
            "pkv_rope_qk",
            _lib.load().pkv_rope_qk(q.data_ptr(), k.data_ptr(), cos.data_ptr(), sin.data_ptr(), qo.data_ptr(),
                                    ko.data_ptr(), rows, num_q_heads, num_kv_heads, head_dim, q.stride(0),
                                    k.stride(0), cos.stride(0), num_q_heads * head_dim, k_rows,
                                    _dtype_code(q, "q"), _stream(dev)),
        )
    return qo, ko


# ---------------------------------------------------------------------------
# sampling
# ---------------------------------------------------------------------------
# ---------------------------------------------------------------------------
# projections of the decode step (tcgen05 GEMM)
# ---------------------------------------------------------------------------
def linear_supported(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """Whether linear() serves these operands: CUDA bf16 / fp16 x and weight of
    one dtype, in_features a multiple of 64, 16-byte aligned rows with
    contiguous columns."""
    return (x.is_cuda and weight.is_cuda and x.dtype == weight.dtype and x.dtype in (torch.bfloat16, torch.float16)
            and x.ndim == 2 and weight.ndim == 2 and x.shape[1] == weight.shape[1] and x.shape[1] % 64 == 0
            and x.stride(1) == 1 and weight.stride(1) == 1 and x.stride(0) % 8 == 0 and weight.stride(0) % 8 == 0
            and x.data_ptr() % 16 == 0 and weight.data_ptr() % 16 == 0)


def linear(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    *,
    out: Optional[torch.Tensor] = None,
    silu_gate: bool = False,
    weight_up: Optional[torch.Tensor] = None,
    status: Optional[torch.Tensor] = None,
    weights_static: bool = False,
) -> torch.Tensor:
    """``x @ weight.T (+ bias)`` for the few activation rows of a decode step,
    on the tcgen05 tensor cores (C ABI pkv_linear): x [rows, K], weight in
    nn.Linear's [N, K] layout, fp32 accumulation, output in x's dtype.

    silu_gate=True: weight is the gate_proj weight [n, K] and weight_up the
    up_proj weight (or, without weight_up, weight is the two stacked, [2 n, K]);
    the result [rows, n] is ``silu(x @ gate.T) * (x @ up.T)`` with the rounding
    of HF Qwen2MLP (each GEMM output, the activation and the product rounded to
    the dtype). Rows beyond 128 run as further launches of 128 rows.

    weights_static=True promises that no kernel still queued on the stream
    writes weight / weight_up (model weights during generation): the launch
    then streams its first weight tiles while the previous kernel finishes.
    """
    if not linear_supported(x, weight):
        raise ValueError("linear needs CUDA bf16/fp16 x [rows, K] and weight [N, K] of one dtype, K a multiple of "
                         "64, contiguous 16-byte aligned rows.")
    dev = _require_cuda(x, weight, bias, out, status, weight_up)
    rows, k = x.shape
    if weight_up is not None:
        if not silu_gate or weight_up.shape != weight.shape or weight_up.stride() != weight.stride() \
                or weight_up.dtype != weight.dtype or weight_up.data_ptr() % 16 != 0:
            raise ValueError("weight_up must match weight (shape, strides, dtype) and needs silu_gate.")
        n = weight.shape[0]
    else:
        n = weight.shape[0] // 2 if silu_gate else weight.shape[0]
    if silu_gate and ((weight_up is None and weight.shape[0] % 2 != 0) or bias is not None):
        raise ValueError("silu_gate needs gate / up weights (separate, or stacked [2 n, K]) and no bias.")
    if bias is not None and (bias.dtype != x.dtype or bias.numel() != n or bias.stride(0) != 1):
        raise ValueError("bias must be a contiguous [N] tensor of x's dtype.")
    if out is None:
        out = torch.empty(rows, n, dtype=x.dtype, device=dev)
    elif out.dtype != x.dtype or tuple(out.shape) != (rows, n) or out.stride(1) != 1:
        raise ValueError(f"out must be a [rows, {n}] tensor of x's dtype with contiguous rows.")
    lib = _lib.load()
    act = _lib.LINEAR_SILU_GATE if silu_gate else _lib.LINEAR_NONE
    if weights_static:
        act |= _lib.LINEAR_WEIGHTS_STATIC
    code = _dtype_code(x, "x")
    with _device_ctx(dev):
        st = _stream(dev)
        for r0 in range(0, rows, 128):
            r = min(128, rows - r0)
            _lib.check("pkv_linear", lib.pkv_linear(
                x[r0:].data_ptr(), weight.data_ptr(), _lib.ptr(weight_up), _lib.ptr(bias), out[r0:].data_ptr(), r, n,
                k, x.stride(0), weight.stride(0), out.stride(0), code, act, _status_ptr(status), st))
    return out


def sample_top_p(
    logits: torch.Tensor,
    temperature: float,
    top_p: float,
    generator: Optional[torch.Generator] = None,
    force_radix: bool = False,
) -> torch.Tensor:
    """One token per row of logits [B, V]: temperature + nucleus (top-p) sampling.

    The nucleus is the reference's (paged_kv.py:418-450): softmax(logits / T)
    in descending order, tokens kept while their running probability stays
    <= top_p, the most likely token always kept; top_p >= 1 keeps all. One
    launch per call (C ABI pkv_sample_top_p) instead of a sort of the whole
    vocabulary. The draw uses one uniform per row from ``generator`` (so a
    seeded generator reproduces the tokens) and the inverse CDF of the kept
    tokens in index order. Returns int64 [B]. ``force_radix`` selects the
    radix-select path for 16-bit logits (the same tokens, slower).
    """
    if logits.ndim != 2:
        raise ValueError(f"logits must be [batch, vocab], got {tuple(logits.shape)}.")
    if not temperature > 0.0 or not top_p > 0.0:
        raise ValueError("temperature and top_p must be > 0 for sampling.")
    dev = _require_cuda(logits)
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    batch, vocab = logits.shape
    u = torch.rand(batch, device=dev, dtype=torch.float32, generator=generator)
    out = torch.empty(batch, dtype=torch.int64, device=dev)
    lib = _lib.load()
    with _device_ctx(dev):
        _lib.check(
            "pkv_sample_top_p",
            lib.pkv_sample_top_p(logits.data_ptr(), _dtype_code(logits, "logits"), batch, vocab, logits.stride(0),
                                 float(max(temperature, 1e-6)), float(top_p if top_p < 1.0 else 2.0),
                                 u.data_ptr(), out.data_ptr(), _lib.SAMPLE_FORCE_RADIX if force_radix else 0,
                                 _stream(dev)),
        )
    return out


def decode_kernel_kind(q: torch.Tensor, k_cache: torch.Tensor, force_generic: bool = False) -> str:
    """'tensor_core' or 'cuda_core': which decode kernel these tensors select."""
    hq, head_dim = q.shape[1], q.shape[2]
    _, hkv, block_size, _ = k_cache.shape
    kind = _lib.check(
        "pkv_decode_kernel_kind",
        _lib.load().pkv_decode_kernel_kind(
            k_cache.data_ptr(), hq, hkv, head_dim, block_size, _strides(k_cache.stride()),
            _dtype_code(q, "q"), _dtype_code(k_cache, "k_cache"),
            _lib.DECODE_FORCE_GENERIC if force_generic else 0,
        ),
    )
    return "tensor_core" if kind == 1 else "cuda_core"
