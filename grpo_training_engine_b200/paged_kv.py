"""Paged-KV rollout decoding with the reference's Python signatures.

Drop-in for src/triton_kernels/paged_kv.py: ``paged_kv_decode`` (low-level,
caller-owned cache and closures, paged_kv.py:840-985) and
``paged_kv_decode_model`` (HF Qwen2-style model, paged_kv.py:589-837). The
KV page append and the decode attention run in libpkv.so (sm_100a CUDA); the
per-token model glue (norms, projections, RoPE, MLP, sampling) stays in
torch, as it does in the reference.

Behaviour kept from the reference (same conditions, same messages): input
validation (paged_kv.py:366-415), max_new_tokens > 0, the capacity check,
qkv_proj_fn / logits_fn shape checks, the [B, max_new_tokens] return shape,
finished rows emitting input_ids[:, 0] (low level) or pad_token_id (model
level), context_lens advancing only for unfinished rows (low level) or for
all rows (model level).

Deliberate differences (reference defects, see the design notes):
  D1 the model path gives every row its own pages (the reference shares one
     block table across the micro-batch, paged_kv.py:635-638, so rows
     overwrite each other's appended tokens);
  D3 the model path keeps the grouped-query cache (Hkv heads) instead of
     replicating K/V to Hq heads (paged_kv.py:574-575,723-724);
  D4 the low-level path checks that every step fits the block table up
     front (the reference checks only the first step, paged_kv.py:871-872).
"""

from __future__ import annotations

import math
from typing import Callable, Optional, Tuple, cast

import numpy as np
import torch

from . import ops
from .kv_pool import KVPagePool


# ---------------------------------------------------------------------------
# validation and sampling (same contract as paged_kv.py:366-450)
# ---------------------------------------------------------------------------
def _validate_inputs(
    input_ids: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
) -> Tuple[int, int, int, int]:
    """Shape/device/dtype checks; returns (heads, block_size, head_dim, max_context)."""
    if input_ids.ndim != 2:
        raise ValueError(f"input_ids must be [batch, seq_len], got {input_ids.shape}.")
    if k_cache.ndim != 4 or v_cache.ndim != 4:
        raise ValueError("k_cache/v_cache must be [num_blocks, heads, block, head_dim].")
    if k_cache.shape != v_cache.shape:
        raise ValueError("k_cache and v_cache must have identical shapes.")
    if block_tables.ndim != 2:
        raise ValueError(f"block_tables must be [batch, max_blocks], got {block_tables.shape}.")
    if context_lens.ndim != 1:
        raise ValueError(f"context_lens must be [batch], got {context_lens.shape}.")
    batch_size = input_ids.shape[0]
    if block_tables.shape[0] != batch_size:
        raise ValueError("block_tables batch dimension must match input_ids batch.")
    if context_lens.shape[0] != batch_size:
        raise ValueError("context_lens batch dimension must match input_ids batch.")
    if not (input_ids.is_cuda and k_cache.is_cuda and v_cache.is_cuda):
        raise ValueError("inputs and caches must be on CUDA device.")
    if not block_tables.is_cuda or not context_lens.is_cuda:
        raise ValueError("block_tables and context_lens must be on CUDA device.")
    if k_cache.dtype != torch.bfloat16 or v_cache.dtype != torch.bfloat16:
        raise ValueError("k_cache/v_cache must be bfloat16.")
    _, num_heads, block_size, head_dim = k_cache.shape
    max_context = block_tables.shape[1] * block_size
    return num_heads, block_size, head_dim, max_context


def _apply_top_p(logits: torch.Tensor, top_p: float) -> torch.Tensor:
    """Nucleus filter: keep the sorted tokens whose cumulative probability stays <= top_p.

    The most likely token is always kept; top_p >= 1 keeps everything and
    top_p <= 0 masks everything (the rule of paged_kv.py:418-434).
    """
    if top_p >= 1.0:
        return logits
    if top_p <= 0.0:
        return torch.full_like(logits, -float("inf"))
    ordered, order = torch.sort(logits, dim=-1, descending=True)
    mass = torch.softmax(ordered, dim=-1).cumsum(dim=-1)
    drop = mass > top_p
    drop[..., 0] = False  # the most likely token always survives
    kept = torch.full_like(logits, -float("inf"))
    return kept.scatter(-1, order, ordered.masked_fill(drop, -float("inf")))


def _sample_tokens(
    logits: torch.Tensor,
    do_sample: bool,
    temperature: float,
    top_p: float,
    generator: Optional[torch.Generator],
) -> torch.Tensor:
    """Greedy when not sampling (or temperature <= 0), else temperature + top-p multinomial.

    CUDA logits with top_p > 0 go through one launch of the sampling kernel
    (ops.sample_top_p) instead of a sort of the vocabulary.
    """
    if not do_sample or temperature <= 0.0:
        return torch.argmax(logits, dim=-1)
    if logits.is_cuda and top_p > 0.0:
        return ops.sample_top_p(logits, temperature, top_p, generator)
    probs = torch.softmax(_apply_top_p(logits / max(temperature, 1e-6), top_p), dim=-1)
    return torch.multinomial(probs, num_samples=1, generator=generator).squeeze(-1)


def _make_generator(device: torch.device, seed: Optional[int]) -> Optional[torch.Generator]:
    if seed is None:
        return None
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    return gen


# ---------------------------------------------------------------------------
# low-level decode loop (paged_kv.py:840-985)
# ---------------------------------------------------------------------------
@torch.no_grad()
def paged_kv_decode(
    input_ids: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    qkv_proj_fn: Callable[[torch.Tensor], Tuple[torch.Tensor, torch.Tensor, torch.Tensor]],
    logits_fn: Callable[[torch.Tensor], torch.Tensor],
    max_new_tokens: int = 128,
    temperature: float = 1.0,
    top_p: float = 1.0,
    do_sample: bool = True,
    eos_token_id: Optional[int] = None,
    pad_token_id: Optional[int] = None,
    seed: Optional[int] = None,
    attention_mask: Optional[torch.Tensor] = None,
    use_cache: Optional[bool] = None,
) -> torch.Tensor:
    """Autoregressive decode over a caller-owned paged cache; returns [B, max_new_tokens].

    Each step: q, k_new, v_new = qkv_proj_fn(last_tokens) ([B, H, D], with H
    the cache heads or any multiple of them for grouped-query models); the
    new K/V go to position context_lens[b]; unfinished rows advance
    context_lens; attention over the pages gives fp32 [B, H, D] for
    logits_fn. attention_mask and use_cache are accepted and ignored, as in
    the reference.
    """
    if max_new_tokens <= 0:
        raise ValueError(f"max_new_tokens must be > 0, got {max_new_tokens}.")
    num_heads, block_size, head_dim, max_context = _validate_inputs(
        input_ids, k_cache, v_cache, block_tables, context_lens
    )
    if context_lens.max().item() >= max_context:
        raise ValueError("context_lens exceed block table capacity.")
    if context_lens.max().item() + max_new_tokens > max_context:
        raise ValueError("context_lens + max_new_tokens exceed block table capacity.")
    eos = -1 if eos_token_id is None else eos_token_id
    pad = 0 if pad_token_id is None else pad_token_id

    batch_size = input_ids.shape[0]
    device = input_ids.device
    generated = torch.full((batch_size, max_new_tokens), pad, device=device, dtype=input_ids.dtype)
    generator = _make_generator(device, seed)
    last_tokens = input_ids[:, -1]
    finished = torch.zeros(batch_size, device=device, dtype=torch.bool)
    context_lens = context_lens.to(torch.int32)
    block_tables = block_tables.to(torch.int32)
    scale = 1.0 / math.sqrt(head_dim)

    any_finished = False
    # without an EOS id no row ever finishes, so the reference's per-step
    # finished.all() check (a host sync) always reads False and is skipped
    track_finished = eos >= 0
    for step in range(max_new_tokens):
        if step and track_finished:
            # one host sync per step, as the reference's finished.all() check
            all_done, any_finished = torch.stack([finished.all(), finished.any()]).tolist()
            if all_done:
                break
        q, k_new, v_new = qkv_proj_fn(last_tokens)
        if q.ndim != 3 or q.shape[0] != batch_size or q.shape[2] != head_dim or q.shape[1] % num_heads != 0:
            raise ValueError("qkv_proj_fn must return [B, H, D] tensors.")
        q = q.to(dtype=torch.bfloat16)
        k_new = k_new.to(dtype=torch.bfloat16)
        v_new = v_new.to(dtype=torch.bfloat16)
        if k_new.stride() != v_new.stride():
            v_new = v_new.contiguous()
            k_new = k_new.contiguous()
        if not any_finished:
            # every row advances: append at the pre-step length and attend over
            # one more, in one launch (pkv_append_decode_run)
            context_lens = context_lens + 1
            attn_out = ops.paged_attention_decode(q, k_cache, v_cache, block_tables, context_lens, scale=scale,
                                                  k_new=k_new, v_new=v_new)
        else:
            # finished rows write their token past their (unchanged) length, as
            # the reference does (paged_kv.py:914-938): append, then decode
            ops.paged_kv_append(k_new, v_new, k_cache, v_cache, block_tables, context_lens)
            context_lens = context_lens + (~finished).to(context_lens.dtype)
            attn_out = ops.paged_attention_decode(q, k_cache, v_cache, block_tables, context_lens, scale=scale)
        logits = logits_fn(attn_out)
        if logits.ndim != 2 or logits.shape[0] != batch_size:
            raise ValueError("logits_fn must return [B, vocab] logits.")
        next_tokens = _sample_tokens(logits, do_sample, temperature, top_p, generator)
        if track_finished:
            next_tokens = torch.where(finished, input_ids[:, 0], next_tokens)
        generated[:, step] = next_tokens
        last_tokens = next_tokens
        if track_finished:
            finished = finished | (next_tokens == eos)
    return generated


# ---------------------------------------------------------------------------
# model-level decode (paged_kv.py:453-837)
# ---------------------------------------------------------------------------
def _first_attr(objs, names):
    for obj in objs:
        if obj is None:
            continue
        for n in names:
            v = getattr(obj, n, None)
            if v is not None:
                return v
    return None


def _get_model_components(model: torch.nn.Module):
    """(embed, layers, norm, rotary_emb, lm_head, Hq, Hkv, head_dim, hidden) of an HF decoder."""
    root = getattr(model, "model", None) or model
    for attr in ("embed_tokens", "layers", "norm", "rotary_emb"):
        if not hasattr(root, attr):
            raise AttributeError(f"Model missing {attr} for paged_kv_decode.")
    if not hasattr(model, "lm_head"):
        raise AttributeError("Model missing lm_head for paged_kv_decode.")
    config = getattr(model, "config", None)
    num_heads = _first_attr([model, config], ["num_heads", "n_heads", "num_attention_heads"])
    if num_heads is None:
        raise ValueError("Unable to infer num_heads for paged_kv_decode.")
    num_kv_heads = _first_attr([model, config], ["num_kv_heads", "n_kv_heads", "num_key_value_heads"])
    if num_kv_heads is None:
        raise ValueError("Unable to infer num_kv_heads for paged_kv_decode.")
    hidden = _first_attr([model, config], ["hidden_size", "embed_dim"])
    if hidden is None:
        raise ValueError("Unable to infer hidden_size for paged_kv_decode.")
    head_dim = _first_attr([model, config], ["head_dim", "attention_head_size"])
    if head_dim is None:
        head_dim = int(hidden) // int(num_heads)
    num_heads, num_kv_heads = int(num_heads), int(num_kv_heads)
    if num_heads % num_kv_heads != 0:
        raise ValueError(f"num_heads ({num_heads}) must be divisible by num_kv_heads ({num_kv_heads}).")
    return (root.embed_tokens, list(root.layers), root.norm, root.rotary_emb, model.lm_head,
            num_heads, num_kv_heads, int(head_dim), int(hidden))


def _layer_kv(past_kv, layer_idx: int) -> tuple[torch.Tensor, torch.Tensor]:
    layers = getattr(past_kv, "layers", None)
    if layers is not None:
        return layers[layer_idx].keys, layers[layer_idx].values
    k, v = past_kv[layer_idx]
    return k, v


def _prefill_paged_cache(
    model: torch.nn.Module,
    input_ids: torch.Tensor,
    attention_mask: torch.Tensor,
    pool: KVPagePool,
    block_tables: torch.Tensor,
) -> None:
    """HF forward over the prompt (minus its last token), then one bulk page write per layer.

    Replaces the reference's B x T x L loop of slice assignments with
    ``.item()`` syncs (paged_kv.py:547-586) by one append_prompt launch per
    layer, in the grouped-query layout (no repeat_kv).
    """
    if input_ids.numel() == 0:
        return
    outputs = model.model(input_ids=input_ids, attention_mask=attention_mask, use_cache=True)
    past_kv = outputs.past_key_values
    if past_kv is None:
        return
    for layer_idx in range(pool.num_layers):
        k_layer, v_layer = _layer_kv(past_kv, layer_idx)
        k_cache, v_cache = pool.layer(layer_idx)
        k_layer = k_layer.to(k_cache.dtype)
        v_layer = v_layer.to(k_cache.dtype)
        if k_layer.stride() != v_layer.stride():
            k_layer, v_layer = k_layer.contiguous(), v_layer.contiguous()
        ops.paged_kv_append_prompt(k_layer, v_layer, k_cache, v_cache, block_tables)


def _prompt_groups(prompt_ids: torch.Tensor, prompt_mask: torch.Tensor) -> list[int]:
    """Group id of each row: the first row with the same prompt tokens and mask."""
    if prompt_ids.shape[0] > 1 and prompt_ids.stride(0) == 0 and prompt_mask.stride(0) == 0:
        return [0] * prompt_ids.shape[0]  # one prompt expanded to the batch
    key = torch.cat([prompt_ids.long(), prompt_mask.long()], dim=1).cpu().numpy()
    _, first, inverse = np.unique(key, axis=0, return_index=True, return_inverse=True)
    return first[inverse.reshape(-1)].tolist()


@torch.no_grad()
def paged_kv_decode_model(
    model: torch.nn.Module,
    input_ids: torch.Tensor,
    attention_mask: torch.Tensor,
    max_new_tokens: int,
    block_size: int,
    do_sample: bool,
    temperature: float,
    top_p: float,
    pad_token_id: int,
    eos_token_id: Optional[int],
    seed: Optional[int],
    use_cuda_graph: bool = True,
    share_prompt_pages: bool = True,
) -> torch.Tensor:
    """Rollout of an HF Qwen2-style decoder over a paged cache; returns [B, max_new_tokens].

    The prompt minus its last token is prefilled with an HF forward and
    written into pages; each step then embeds the last token, and per layer
    runs norm -> q/k/v projection + RoPE -> page append + paged decode
    attention (one launch) -> o_proj -> MLP, then samples the next token
    (paged_kv.py:690-837).

    With use_cuda_graph (the default), the step's model forward -- embedding,
    every layer, final norm and LM head -- is captured once as a CUDA graph
    after the first (eager) step and replayed for the others, so a step costs
    one launch instead of ~15 per layer from Python; sampling stays eager.
    This is the graph capture the reference leaves disabled
    (``use_cuda_graph = False``, paged_kv.py:687). A model whose forward
    cannot be captured falls back to eager steps; the tokens are identical
    either way (the same kernels run on the same buffers).

    With share_prompt_pages (the default), rows whose prefilled prompts are
    identical -- a GRPO group, which the trainer passes as one prompt
    expanded to the micro-batch (trainer.py:389-392) -- are prefilled once:
    one HF forward per distinct prompt, its full pages shared by reference
    count and only the partially filled last prompt page copied per row, the
    paged form of the trainer's prefix expansion (trainer.py:465-484).
    Decode then reads a group's prompt pages from L2 after the first row.
    """
    if max_new_tokens <= 0:
        raise ValueError(f"max_new_tokens must be > 0, got {max_new_tokens}.")
    (embeddings, layers, norm, rotary_emb, lm_head, num_heads, num_kv_heads, head_dim, _) = (
        _get_model_components(model)
    )
    batch_size, prompt_len = input_ids.shape
    if prompt_len == 0:
        raise ValueError("input_ids must have at least 1 token.")
    device = input_ids.device
    max_context_needed = max(prompt_len - 1 + max_new_tokens + 1, 1)
    pages_per_seq = math.ceil(max_context_needed / block_size)

    prefix = prompt_len - 1
    groups = _prompt_groups(input_ids[:, :-1], attention_mask[:, :-1]) \
        if share_prompt_pages and batch_size > 1 and prefix > 0 else list(range(batch_size))
    pool = KVPagePool(KVPagePool.pages_needed_shared(groups, prefix, max_context_needed, block_size),
                      len(layers), num_kv_heads, block_size, head_dim, dtype=torch.bfloat16, device=device)
    tables, reps = pool.share_prompts(groups, prefix, max_context_needed)
    block_tables = pool.block_table(tables, width=pages_per_seq)
    context_lens = torch.full((batch_size,), prefix, device=device, dtype=torch.int32)
    if prefix > 0:
        if len(reps) == batch_size:
            _prefill_paged_cache(model, input_ids[:, :-1], attention_mask[:, :-1], pool, block_tables)
        else:
            rep_idx = torch.as_tensor(reps, device=device)
            _prefill_paged_cache(model, input_ids[rep_idx, :-1], attention_mask[rep_idx, :-1], pool,
                                 block_tables[rep_idx])
            pool.copy_prefix_tails(tables, groups, prefix)

    generated = torch.full((batch_size, max_new_tokens), pad_token_id, device=device, dtype=input_ids.dtype)
    generator = _make_generator(device, seed)
    finished = torch.zeros(batch_size, device=device, dtype=torch.bool)
    scale = 1.0 / math.sqrt(head_dim)
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

    # The forward reads the step's inputs from fixed buffers (the last tokens
    # and the pre-append context lengths), so a CUDA graph of it can be
    # replayed with new values; its outputs are the logits and the post-append
    # lengths.
    tokens_buf = input_ids[:, -1].clone()
    ctx_buf = context_lens
    plan_ws = ops.plan_decode(ctx_buf + 1, num_heads, num_kv_heads, head_dim, block_size,
                              block_tables.shape[1]).workspace

    # The element-wise steps around the projections (residual add + RMSNorm,
    # RoPE of the new q / k rows) run as one launch each (ops.add_rmsnorm,
    # ops.rope_qk) for a bf16 model (the cache dtype) whose norms are plain
    # weight-scaled RMSNorms; otherwise through the model's own modules.
    norms = [norm] + [m for layer in layers for m in (layer.input_layernorm, layer.post_attention_layernorm)]
    fused_glue = all(
        isinstance(getattr(m, "weight", None), torch.Tensor) and getattr(m, "variance_epsilon", None) is not None
        and m.weight.dtype == embeddings.weight.dtype and m.weight.ndim == 1 and m.weight.numel() <= 4096
        for m in norms) and head_dim % 2 == 0 and embeddings.weight.dtype == torch.bfloat16 \
        and embeddings.weight.shape[1] % 8 == 0
    # a plain SiLU-gated MLP: its activation and product run as one launch (ops.silu_mul)
    silu_mlp = all(type(getattr(layer.mlp, "act_fn", None)).__name__ in ("SiLUActivation", "SiLU")
                   and all(hasattr(layer.mlp, n) for n in ("gate_proj", "up_proj", "down_proj"))
                   and layer.mlp.gate_proj.out_features % 8 == 0 for layer in layers)

    # Projections that read the same input run as one GEMM on stacked weights:
    # q / k / v (with their biases) and the MLP's gate / up. Every projection of
    # the fused path multiplies by a transposed (input-major) copy of its
    # weights, for which cuBLAS picks faster kernels at this batch size (7-18%
    # per GEMM on B200 at 128 rows). The copies are made from the modules'
    # current weights for this call (the trainer updates them between
    # rollouts); modules that are not plain nn.Linear (e.g. LoRA-wrapped) are
    # called as they are.
    def _stack(mods):
        if not all(type(m) is torch.nn.Linear for m in mods):
            return None
        wt = torch.cat([m.weight.detach() for m in mods], 0).t().contiguous()
        if all(m.bias is None for m in mods):
            return wt, None
        return wt, torch.cat([m.bias.detach() if m.bias is not None else
                              torch.zeros(m.out_features, dtype=wt.dtype, device=wt.device) for m in mods])

    def _linear(st, mod, h):
        if st is None:
            return mod(h)
        return h @ st[0] if st[1] is None else torch.addmm(st[1], h, st[0])

    # The MLP's projections run on the tcgen05 projection kernel (ops.linear)
    # straight from the modules' own weights: gate and up with the SiLU gate in
    # one launch, then down. Plain bias-free 16-bit nn.Linear modules with
    # in_features a multiple of 64 (every Qwen2 MLP); no copies are made. The
    # weights do not change during generation, so each launch starts
    # streaming them while the previous kernel finishes (weights_static).
    # q / k / v, o_proj and the LM head stay on cuBLAS: on pkv_linear the
    # first two made the 1.5B rollout step ~4% slower (their ~6 MB of weights
    # take less time than each CTA's re-read of the activation rows and the
    # split-K reduction), and the LM head's 150k columns are ~4 waves of
    # 256-column tiles whose short last wave costs more than cuBLAS's schedule.
    def _tc_mlp_ok(mlp) -> bool:
        mods = [getattr(mlp, n, None) for n in ("gate_proj", "up_proj", "down_proj")]
        return all(type(m) is torch.nn.Linear and m.bias is None and m.weight.dtype == embeddings.weight.dtype
                   and m.weight.dtype in (torch.bfloat16, torch.float16) and m.weight.is_cuda
                   and m.weight.is_contiguous() and m.in_features % 64 == 0 and m.weight.data_ptr() % 16 == 0
                   for m in mods) \
            and mods[0].out_features % 64 == 0 and mods[0].weight.shape == mods[1].weight.shape
    tc_mlp = [bool(fused_glue and silu_mlp and _tc_mlp_ok(layer.mlp)) for layer in layers]

    # the copies need as much memory as those weights; without twice that free
    # (the trainer may hold most of the GPU) the modules are called as they are
    proj_bytes = sum(m.weight.numel() * m.weight.element_size() for i, layer in enumerate(layers)
                     for owner, names in ((layer.self_attn, ("q_proj", "k_proj", "v_proj", "o_proj")),
                                          (layer.mlp, () if tc_mlp[i] else ("gate_proj", "up_proj", "down_proj")))
                     for m in (getattr(owner, n, None) for n in names)
                     if isinstance(getattr(m, "weight", None), torch.Tensor)) if fused_glue else 0
    if fused_glue and device.type == "cuda" and torch.cuda.mem_get_info(device)[0] < 2 * proj_bytes:
        fused_glue_copies = False
    else:
        fused_glue_copies = fused_glue
    qkv_stack = [_stack((layer.self_attn.q_proj, layer.self_attn.k_proj, layer.self_attn.v_proj))
                 if fused_glue_copies else None for layer in layers]
    o_stack = [_stack((layer.self_attn.o_proj,)) if fused_glue_copies else None for layer in layers]
    gate_up_stack = [_stack((layer.mlp.gate_proj, layer.mlp.up_proj))
                     if fused_glue_copies and silu_mlp and not tc_mlp[i] else None for i, layer in enumerate(layers)]
    down_stack = [_stack((layer.mlp.down_proj,)) if fused_glue_copies and silu_mlp and not tc_mlp[i] else None
                  for i, layer in enumerate(layers)]
    head_stack = _stack((lm_head,)) if fused_glue_copies else None
    q_cols, kv_cols = num_heads * head_dim, num_kv_heads * head_dim
    # With stacked q / k / v on the tensor-core decode, RoPE runs inside the
    # decode launch (ops.paged_attention_decode(rope=...)): q and k are passed
    # as the projection wrote them, and the separate RoPE launch disappears.
    rope_in_decode = fused_glue and all(st is not None for st in qkv_stack) and ops.decode_kernel_kind(
        torch.empty(batch_size, num_heads, head_dim, dtype=pool.k.dtype, device=device),
        pool.layer(0)[0]) == "tensor_core" and head_dim % 16 == 0

    def _qkv(layer_idx, attn, h):
        st = qkv_stack[layer_idx]
        if st is None:
            return attn.q_proj(h), attn.k_proj(h), attn.v_proj(h)
        qkv = _linear(st, None, h)
        return qkv[:, :q_cols], qkv[:, q_cols:q_cols + kv_cols], qkv[:, q_cols + kv_cols:]

    def _mlp(layer_idx, layer, h):
        mlp = layer.mlp
        if not silu_mlp:
            return mlp(h)
        if tc_mlp[layer_idx] and ops.linear_supported(h, mlp.gate_proj.weight):
            act = ops.linear(h, mlp.gate_proj.weight, silu_gate=True, weight_up=mlp.up_proj.weight,
                             weights_static=True)
            return ops.linear(act, mlp.down_proj.weight, weights_static=True)
        st = gate_up_stack[layer_idx]
        if st is None:
            return _linear(down_stack[layer_idx], mlp.down_proj, ops.silu_mul(mlp.gate_proj(h), mlp.up_proj(h)))
        inter = mlp.gate_proj.out_features
        gu = _linear(st, None, h)
        return _linear(down_stack[layer_idx], mlp.down_proj, ops.silu_mul(gu[:, :inter], gu[:, inter:]))

    def _forward_modules() -> tuple[torch.Tensor, torch.Tensor]:
        hidden = cast(torch.Tensor, embeddings(tokens_buf))
        if hidden.ndim == 2:
            hidden = hidden.unsqueeze(1)
        cos, sin = rotary_emb(hidden, ctx_buf.unsqueeze(1))
        new_context_lens = ctx_buf + 1
        plan = ops.plan_decode(new_context_lens, num_heads, num_kv_heads, head_dim, block_size,
                               block_tables.shape[1], workspace=plan_ws)
        for layer_idx, layer in enumerate(layers):
            attn = layer.self_attn
            residual = hidden
            h = layer.input_layernorm(hidden)
            q = attn.q_proj(h).view(batch_size, 1, num_heads, head_dim).transpose(1, 2)
            k = attn.k_proj(h).view(batch_size, 1, num_kv_heads, head_dim).transpose(1, 2)
            v = attn.v_proj(h).view(batch_size, 1, num_kv_heads, head_dim).transpose(1, 2)
            q, k = apply_rotary_pos_emb(q, k, cos, sin)
            q1 = q[:, :, 0, :].to(torch.bfloat16)
            k1 = k[:, :, 0, :].to(torch.bfloat16).contiguous()
            v1 = v[:, :, 0, :].to(torch.bfloat16).contiguous()
            k_cache, v_cache = pool.layer(layer_idx)
            # append at context_lens and attend over new_context_lens: one fused call
            attn_out = ops.paged_attention_decode(q1, k_cache, v_cache, block_tables, new_context_lens,
                                                  scale=scale, plan=plan, k_new=k1, v_new=v1,
                                                  early_start=layer_idx > 0)
            attn_out = attn_out.to(hidden.dtype).reshape(batch_size, 1, num_heads * head_dim)
            hidden = residual + attn.o_proj(attn_out)
            residual = hidden
            hidden = residual + layer.mlp(layer.post_attention_layernorm(hidden))
        hidden = norm(hidden)
        return lm_head(hidden[:, -1, :]), new_context_lens

    def _forward_fused() -> tuple[torch.Tensor, torch.Tensor]:
        hidden = cast(torch.Tensor, embeddings(tokens_buf))  # [B, hidden]
        cos, sin = rotary_emb(hidden.unsqueeze(1), ctx_buf.unsqueeze(1))
        cos, sin = cos.reshape(batch_size, head_dim), sin.reshape(batch_size, head_dim)
        new_context_lens = ctx_buf + 1
        plan = ops.plan_decode(new_context_lens, num_heads, num_kv_heads, head_dim, block_size,
                               block_tables.shape[1], workspace=plan_ws)
        pending = None  # the previous layer's MLP output, added in the next norm
        for layer_idx, layer in enumerate(layers):
            attn = layer.self_attn
            ln = layer.input_layernorm
            h, total = ops.add_rmsnorm(hidden if pending is None else pending, ln.weight, ln.variance_epsilon,
                                       residual=None if pending is None else hidden)
            if total is not None:
                hidden = total
            q_lin, k_lin, v_lin = _qkv(layer_idx, attn, h)
            k_cache, v_cache = pool.layer(layer_idx)
            v1 = v_lin.view(batch_size, num_kv_heads, head_dim)
            # every layer after the first: the last kernel before the plan, block tables and this layer's
            # cache changed is the previous layer's decode launch, so this one may schedule its pages early
            early = layer_idx > 0
            if rope_in_decode:
                # RoPE, append at context_lens and attention over new_context_lens: one launch
                attn_out = ops.paged_attention_decode(
                    q_lin.view(batch_size, num_heads, head_dim), k_cache, v_cache, block_tables,
                    new_context_lens, scale=scale, plan=plan, k_new=k_lin.view(batch_size, num_kv_heads, head_dim),
                    v_new=v1, rope=(cos, sin), out_dtype=hidden.dtype, early_start=early)
            else:
                # stacked: the keys rotate in place, so k and v are views of one buffer with equal strides
                q1, k1 = ops.rope_qk(q_lin, k_lin, cos, sin, num_heads, num_kv_heads, head_dim,
                                     k_out=k_lin if qkv_stack[layer_idx] is not None else None)
                # append at context_lens and attend over new_context_lens: one fused call
                attn_out = ops.paged_attention_decode(q1, k_cache, v_cache, block_tables, new_context_lens,
                                                      scale=scale, plan=plan, k_new=k1, v_new=v1,
                                                      out_dtype=hidden.dtype, early_start=early)
            o = _linear(o_stack[layer_idx], attn.o_proj, attn_out.reshape(batch_size, num_heads * head_dim))
            ln = layer.post_attention_layernorm
            h2, hidden = ops.add_rmsnorm(o, ln.weight, ln.variance_epsilon, residual=hidden)
            pending = _mlp(layer_idx, layer, h2)
        h, _ = ops.add_rmsnorm(pending, norm.weight, norm.variance_epsilon, residual=hidden)
        return _linear(head_stack, lm_head, h), new_context_lens

    _forward = _forward_fused if fused_glue else _forward_modules

    graph: Optional[torch.cuda.CUDAGraph] = None
    graph_out: Optional[tuple[torch.Tensor, torch.Tensor]] = None
    for step in range(max_new_tokens):
        if finished.all():
            break
        if graph is not None:
            graph.replay()
            logits, new_context_lens = graph_out
        else:
            logits, new_context_lens = _forward()
        next_tokens = _sample_tokens(logits, do_sample, temperature, top_p, generator)
        next_tokens = torch.where(finished, torch.full_like(next_tokens, pad_token_id), next_tokens)
        generated[:, step] = next_tokens
        if eos_token_id is not None and eos_token_id >= 0:
            finished = finished | (next_tokens == eos_token_id)
        tokens_buf.copy_(next_tokens)
        ctx_buf.copy_(new_context_lens)
        if step == 0 and use_cuda_graph and device.type == "cuda" and max_new_tokens > 1:
            # the eager first step was the warm-up; capture the forward for the rest
            graph, graph_out = _capture_forward(_forward)
    return generated


def _capture_forward(forward):
    """CUDA graph of forward() and its output tensors, or (None, None) if it cannot be captured."""
    graph = torch.cuda.CUDAGraph()
    try:
        with torch.cuda.graph(graph):
            out = forward()
    except RuntimeError:
        torch.cuda.synchronize()
        return None, None
    return graph, out


__all__ = ["paged_kv_decode", "paged_kv_decode_model"]
