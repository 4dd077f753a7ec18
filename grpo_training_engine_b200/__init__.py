"""B200-native paged-KV rollout path for the GRPO trainer.

Drop-in for the paged-decode entry of ``src.triton_kernels`` (the dispatch
façade at src/triton_kernels/__init__.py:218-297): same function name, same
arguments, same routing between the low-level path (caller-owned cache and
closures) and the model-level path. The page append and decode attention
are hand-written sm_100a CUDA kernels in ``libpkv.so`` behind a C ABI
(include/pkv.h); there is no Triton and no non-CUDA implementation.

``TRITON_AVAILABLE`` keeps the name the trainer reads
(src/grpo/trainer.py:33,387): it is True when the accelerated paged path can
be used (libpkv.so loads), False otherwise — exactly the condition under
which the trainer picks the paged path over HF ``generate``.
"""

from __future__ import annotations

from typing import cast

import torch

from . import _lib
from .kv_pool import KVPagePool, PoolExhausted
from .ops import (
    DecodePlan,
    decode_kernel_kind,
    decode_workspace_bytes,
    gather_kv,
    paged_attention_decode,
    paged_kv_append,
    paged_kv_append_prompt,
    plan_decode,
)
from .paged_kv import paged_kv_decode as _paged_kv_decode_low_level
from .paged_kv import paged_kv_decode_model

try:
    _lib.load()
    PAGED_KV_AVAILABLE = True
    _LOAD_ERROR = ""
except ImportError as _exc:  # library not built
    PAGED_KV_AVAILABLE = False
    _LOAD_ERROR = str(_exc)

TRITON_AVAILABLE = PAGED_KV_AVAILABLE

_LOW_LEVEL_ARGS = ("k_cache", "v_cache", "block_tables", "context_lens", "qkv_proj_fn", "logits_fn")


def paged_kv_decode(model, input_ids, attention_mask=None, max_new_tokens: int = 128, **kwargs):
    """Paged rollout decode with the reference façade's routing.

    With all of ``k_cache, v_cache, block_tables, context_lens, qkv_proj_fn,
    logits_fn`` in kwargs it runs the low-level loop; otherwise it treats
    ``model`` as an HF decoder, left-trims the prompt to the longest real
    length and runs the model-level loop with block_size (default 16),
    do_sample, temperature, top_p, pad_token_id (0), eos_token_id and seed.
    Raises ImportError when libpkv.so is unavailable, like the reference when
    Triton is missing (the trainer falls back to HF generate on it).

    Like the reference, it returns only the new tokens, [B, max_new_tokens]
    (paged_kv.py:662-667). The trainer slices ``outputs[j, prompt_len:]``
    as if it had HF generate's prompt + response rows (trainer.py:444-448);
    ``return_prompt=True`` returns that layout, [B, prompt + max_new_tokens].
    """
    if not PAGED_KV_AVAILABLE:
        raise ImportError(f"paged KV kernels are not available for paged_kv_decode: {_LOAD_ERROR}")
    input_ids_t = cast(torch.Tensor, input_ids)
    return_prompt = bool(kwargs.pop("return_prompt", False))
    out = _route(model, input_ids_t, attention_mask, max_new_tokens, kwargs)
    if return_prompt:
        # HF generate's layout: the prompt as passed, then the new tokens
        return torch.cat([input_ids_t, out.to(input_ids_t.dtype)], dim=1)
    return out


def _route(model, input_ids_t: torch.Tensor, attention_mask, max_new_tokens: int, kwargs: dict):
    mask_t = cast(torch.Tensor, attention_mask) if attention_mask is not None else None
    if all(name in kwargs for name in _LOW_LEVEL_ARGS):
        return _paged_kv_decode_low_level(
            input_ids_t,
            k_cache=kwargs.pop("k_cache"),
            v_cache=kwargs.pop("v_cache"),
            block_tables=kwargs.pop("block_tables"),
            context_lens=kwargs.pop("context_lens"),
            qkv_proj_fn=kwargs.pop("qkv_proj_fn"),
            logits_fn=kwargs.pop("logits_fn"),
            max_new_tokens=max_new_tokens,
            do_sample=kwargs.pop("do_sample", True),
            temperature=kwargs.pop("temperature", 1.0),
            top_p=kwargs.pop("top_p", 1.0),
            pad_token_id=kwargs.pop("pad_token_id", None),
            eos_token_id=kwargs.pop("eos_token_id", None),
            attention_mask=mask_t,
            use_cache=kwargs.pop("use_cache", None),
            **kwargs,
        )

    if mask_t is None:
        prompt_lens = torch.full((input_ids_t.shape[0],), input_ids_t.shape[1], device=input_ids_t.device,
                                 dtype=torch.int32)
    else:
        prompt_lens = mask_t.sum(dim=-1).to(dtype=torch.int32)
    max_prompt_len = int(prompt_lens.max().item()) if prompt_lens.numel() > 0 else 0
    if mask_t is not None and input_ids_t.shape[1] > max_prompt_len:
        input_ids_t = input_ids_t[:, -max_prompt_len:]
        mask_t = mask_t[:, -max_prompt_len:]
    if mask_t is None:
        mask_t = torch.ones_like(input_ids_t, dtype=torch.long)
    return paged_kv_decode_model(
        model=cast(torch.nn.Module, model),
        input_ids=input_ids_t,
        attention_mask=mask_t,
        max_new_tokens=max_new_tokens,
        block_size=int(kwargs.pop("block_size", 16)),
        do_sample=bool(kwargs.pop("do_sample", True)),
        temperature=float(kwargs.pop("temperature", 1.0)),
        top_p=float(kwargs.pop("top_p", 1.0)),
        pad_token_id=int(kwargs.pop("pad_token_id", 0)),
        eos_token_id=kwargs.pop("eos_token_id", None),
        seed=kwargs.pop("seed", None),
        use_cuda_graph=bool(kwargs.pop("use_cuda_graph", True)),
        share_prompt_pages=bool(kwargs.pop("share_prompt_pages", True)),
    )


__all__ = [
    "TRITON_AVAILABLE",
    "PAGED_KV_AVAILABLE",
    "paged_kv_decode",
    "paged_kv_decode_model",
    "paged_kv_append",
    "paged_kv_append_prompt",
    "paged_attention_decode",
    "plan_decode",
    "gather_kv",
    "decode_kernel_kind",
    "decode_workspace_bytes",
    "DecodePlan",
    "KVPagePool",
    "PoolExhausted",
]
