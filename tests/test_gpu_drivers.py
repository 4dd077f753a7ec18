"""The reference-signature drivers on the GPU.

1. The reference's own paged-decode test scenario
   (tests/test_triton_performance.py:136-271): a tiny model decodes greedily
   through the low-level ``paged_kv_decode`` and must produce exactly the
   tokens of a dense fp32 attention reference; run here through this
   package's façade, plus larger batched / grouped-query / shuffled-page
   variants the reference never tests.
2. The model-level path on a tiny random HF Qwen2 decoder: paged rollout vs
   the same step computed with dense K/V tensors.
"""

from __future__ import annotations

import math

import pytest
import torch

import grpo_training_engine_b200 as pkg

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


class TinyPagedModel(torch.nn.Module):
    """Same structure as the reference test model, with optional grouped-query heads."""

    def __init__(self, vocab, num_heads, head_dim, num_kv_heads=None):
        super().__init__()
        self.num_heads, self.head_dim = num_heads, head_dim
        self.num_kv_heads = num_kv_heads or num_heads
        embed = num_heads * head_dim
        self.embed = torch.nn.Embedding(vocab, embed)
        self.q_proj = torch.nn.Linear(embed, embed, bias=False)
        self.k_proj = torch.nn.Linear(embed, self.num_kv_heads * head_dim, bias=False)
        self.v_proj = torch.nn.Linear(embed, self.num_kv_heads * head_dim, bias=False)
        self.out_proj = torch.nn.Linear(embed, vocab, bias=False)

    def _project(self, ids):
        x = self.embed(ids)
        if x.ndim == 2:
            x = x.unsqueeze(1)
        b, s, _ = x.shape
        q = self.q_proj(x).view(b, s, self.num_heads, self.head_dim)
        k = self.k_proj(x).view(b, s, self.num_kv_heads, self.head_dim)
        v = self.v_proj(x).view(b, s, self.num_kv_heads, self.head_dim)
        return q, k, v

    def qkv_for_decode(self, ids):
        q, k, v = self._project(ids)
        return q[:, 0], k[:, 0], v[:, 0]

    def logits_from_attn(self, attn_out):
        return self.out_proj(attn_out.reshape(attn_out.shape[0], -1))

    @torch.no_grad()
    def generate(self, input_ids, max_tokens, return_gaps=False):
        """Dense reference: fp32 softmax attention over bf16-rounded q/K/V.

        With return_gaps, also the top-1 minus top-2 logit gap of every step.
        """
        tokens, out, gaps = input_ids, [], []
        scale = 1.0 / math.sqrt(self.head_dim)
        g = self.num_heads // self.num_kv_heads
        for _ in range(max_tokens):
            q, k, v = self._project(tokens)
            q_last = q[:, -1].to(torch.bfloat16).float()
            k = k.to(torch.bfloat16).float().repeat_interleave(g, dim=2)
            v = v.to(torch.bfloat16).float().repeat_interleave(g, dim=2)
            scores = (q_last[:, None] * k).sum(-1) * scale
            weights = torch.softmax(scores.transpose(1, 2), dim=-1)
            attn = (weights[..., None] * v.transpose(1, 2)).sum(dim=-2)
            logits = self.logits_from_attn(attn)
            nxt = torch.argmax(logits, dim=-1)
            top2 = logits.float().topk(2, dim=-1).values
            gaps.append(top2[:, 0] - top2[:, 1])
            out.append(nxt)
            tokens = torch.cat([tokens, nxt[:, None]], dim=1)
        if return_gaps:
            return torch.stack(out, dim=1), torch.stack(gaps, dim=1)
        return torch.stack(out, dim=1)


def _run_low_level(model, input_ids, block_size, max_new_tokens, shuffle_seed=None):
    batch, prompt_len = input_ids.shape
    max_ctx = prompt_len - 1 + max_new_tokens + 1
    max_blocks = math.ceil(max_ctx / block_size)
    num_blocks = batch * max_blocks
    k_cache = torch.zeros((num_blocks, model.num_kv_heads, block_size, model.head_dim), device=DEV, dtype=torch.bfloat16)
    v_cache = torch.zeros_like(k_cache)
    ids = torch.arange(num_blocks, dtype=torch.int32)
    if shuffle_seed is not None:
        ids = ids[torch.randperm(num_blocks, generator=torch.Generator().manual_seed(shuffle_seed))]
    block_tables = ids.reshape(batch, max_blocks).to(DEV)
    context_lens = torch.full((batch,), prompt_len - 1, device=DEV, dtype=torch.int32)
    if prompt_len > 1:
        with torch.no_grad():
            _, kp, vp = model._project(input_ids[:, :-1])
        # bulk prompt write ([B, H, T, D] layout) instead of the reference's per-position loop
        pkg.paged_kv_append_prompt(kp.transpose(1, 2).to(torch.bfloat16).contiguous(),
                                   vp.transpose(1, 2).to(torch.bfloat16).contiguous(),
                                   k_cache, v_cache, block_tables)
    return pkg.paged_kv_decode(
        None, input_ids=input_ids, k_cache=k_cache, v_cache=v_cache, block_tables=block_tables,
        context_lens=context_lens, qkv_proj_fn=model.qkv_for_decode, logits_fn=model.logits_from_attn,
        max_new_tokens=max_new_tokens, temperature=0.0, top_p=1.0, do_sample=False, eos_token_id=None,
        pad_token_id=0, seed=123,
    )


def test_reference_scenario_token_exact():
    """tests/test_triton_performance.py:136-271 verbatim in its numbers: seed 7, B=1,
    vocab 32, H=2, D=8, prompt 3, 3 new tokens, block size 4."""
    torch.manual_seed(7)
    torch.cuda.manual_seed_all(7)
    model = TinyPagedModel(32, 2, 8).to(DEV)
    input_ids = torch.randint(0, 32, (1, 3), device=DEV)
    got = _run_low_level(model, input_ids, block_size=4, max_new_tokens=3)
    assert torch.equal(got, model.generate(input_ids, 3))


@pytest.mark.parametrize(
    "batch,heads,kv_heads,head_dim,block_size,prompt,new",
    [(4, 2, 2, 8, 4, 5, 8), (3, 12, 2, 128, 16, 40, 24), (2, 28, 4, 128, 16, 19, 12), (5, 4, 1, 64, 16, 1, 6)],
)
def test_batched_gqa_shuffled_pages_token_exact(batch, heads, kv_heads, head_dim, block_size, prompt, new):
    """Greedy tokens equal the dense reference's; the tensor-core path rounds the
    softmax weights to bf16, so a flip is accepted only where the dense logits
    had a near tie (top-2 gap < 0.05) at the first differing step."""
    torch.manual_seed(1000 + batch)
    model = TinyPagedModel(64, heads, head_dim, kv_heads).to(DEV)
    input_ids = torch.randint(0, 64, (batch, prompt), device=DEV)
    got = _run_low_level(model, input_ids, block_size, new, shuffle_seed=batch)
    ref, gaps = model.generate(input_ids, new, return_gaps=True)
    for row in range(batch):
        diff = (got[row] != ref[row]).nonzero()
        if len(diff):
            first = int(diff[0])
            assert float(gaps[row, first]) < 0.05, (row, first, float(gaps[row, first]))


def test_low_level_eos_and_padding_semantics():
    torch.manual_seed(3)
    model = TinyPagedModel(16, 2, 8).to(DEV)
    input_ids = torch.randint(0, 16, (4, 3), device=DEV)
    ref = model.generate(input_ids, 6)
    eos = int(ref[0, 1])
    k_cache = torch.zeros((8, 2, 4, 8), device=DEV, dtype=torch.bfloat16)
    out = pkg.paged_kv_decode(
        None, input_ids=input_ids, k_cache=k_cache, v_cache=torch.zeros_like(k_cache),
        block_tables=torch.arange(8, dtype=torch.int32, device=DEV).reshape(4, 2),
        context_lens=torch.zeros(4, dtype=torch.int32, device=DEV), qkv_proj_fn=model.qkv_for_decode,
        logits_fn=model.logits_from_attn, max_new_tokens=6, do_sample=False, eos_token_id=eos,
    )
    assert out.shape == (4, 6)
    for row in range(4):
        hits = (out[row] == eos).nonzero()
        if len(hits):
            first = int(hits[0])
            # finished rows re-emit input_ids[:, 0] (paged_kv.py:978)
            assert (out[row, first + 1:] == input_ids[row, 0]).all()


def test_low_level_capacity_errors():
    model = TinyPagedModel(16, 2, 8).to(DEV)
    ids = torch.zeros(1, 2, dtype=torch.long, device=DEV)
    kc = torch.zeros((2, 2, 4, 8), device=DEV, dtype=torch.bfloat16)
    common = dict(k_cache=kc, v_cache=kc.clone(), block_tables=torch.zeros(1, 2, dtype=torch.int32, device=DEV),
                  qkv_proj_fn=model.qkv_for_decode, logits_fn=model.logits_from_attn)
    with pytest.raises(ValueError, match="context_lens exceed block table capacity."):
        pkg.paged_kv_decode(None, ids, context_lens=torch.tensor([8], dtype=torch.int32, device=DEV), **common)
    with pytest.raises(ValueError, match="exceed block table capacity"):
        pkg.paged_kv_decode(None, ids, context_lens=torch.tensor([6], dtype=torch.int32, device=DEV),
                            max_new_tokens=4, **common)


# -------------------------------------------------------------- model-level path
def _tiny_qwen2(seed=0):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(seed)
    cfg = Qwen2Config(vocab_size=96, hidden_size=128, intermediate_size=256, num_hidden_layers=3,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=512,
                      rms_norm_eps=1e-6, tie_word_embeddings=False)
    model = Qwen2ForCausalLM(cfg).to(DEV, torch.bfloat16).eval()
    return model


@torch.no_grad()
def _dense_rollout(model, input_ids, max_new_tokens):
    """Same per-step computation as paged_kv_decode_model, with dense K/V tensors."""
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

    m = model.model
    cfg = model.config
    hq, hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    d = cfg.hidden_size // hq
    batch, prompt = input_ids.shape
    out = m(input_ids=input_ids[:, :-1], attention_mask=torch.ones_like(input_ids[:, :-1]), use_cache=True)
    pk = out.past_key_values
    ks = [pk.layers[i].keys.to(torch.bfloat16) for i in range(cfg.num_hidden_layers)]
    vs = [pk.layers[i].values.to(torch.bfloat16) for i in range(cfg.num_hidden_layers)]
    last = input_ids[:, -1]
    pos = prompt - 1
    toks, gaps = [], []
    for _ in range(max_new_tokens):
        h = m.embed_tokens(last).unsqueeze(1)
        cos, sin = m.rotary_emb(h, torch.full((batch, 1), pos, device=DEV))
        for li, layer in enumerate(m.layers):
            a = layer.self_attn
            r = h
            x = layer.input_layernorm(h)
            q = a.q_proj(x).view(batch, 1, hq, d).transpose(1, 2)
            k = a.k_proj(x).view(batch, 1, hkv, d).transpose(1, 2)
            v = a.v_proj(x).view(batch, 1, hkv, d).transpose(1, 2)
            q, k = apply_rotary_pos_emb(q, k, cos, sin)
            ks[li] = torch.cat([ks[li], k.to(torch.bfloat16)], dim=2)
            vs[li] = torch.cat([vs[li], v.to(torch.bfloat16)], dim=2)
            kf = ks[li].float().repeat_interleave(hq // hkv, dim=1)
            vf = vs[li].float().repeat_interleave(hq // hkv, dim=1)
            qf = q.to(torch.bfloat16).float()
            w = torch.softmax((qf @ kf.transpose(-1, -2)) / math.sqrt(d), dim=-1)
            att = (w @ vf).to(h.dtype).transpose(1, 2).reshape(batch, 1, hq * d)
            h = r + a.o_proj(att)
            h = h + layer.mlp(layer.post_attention_layernorm(h))
        logits = model.lm_head(m.norm(h)[:, -1]).float()
        top2 = logits.topk(2, dim=-1).values
        gaps.append(top2[:, 0] - top2[:, 1])
        last = logits.argmax(-1)
        toks.append(last)
        pos += 1
    return torch.stack(toks, 1), torch.stack(gaps, 1)


def test_model_level_matches_dense_rollout():
    model = _tiny_qwen2()
    torch.manual_seed(5)
    input_ids = torch.randint(0, 96, (4, 21), device=DEV)
    got = pkg.paged_kv_decode(model, input_ids, torch.ones_like(input_ids), max_new_tokens=10,
                              do_sample=False, pad_token_id=0)
    ref, gaps = _dense_rollout(model, input_ids, 10)
    assert got.shape == (4, 10)
    for row in range(4):
        diff = (got[row] != ref[row]).nonzero()
        if len(diff):  # only a near-tie in the dense logits may flip a greedy token
            first = int(diff[0])
            assert float(gaps[row, first]) < 0.05, (row, first, float(gaps[row, first]))


@pytest.mark.parametrize("do_sample", [False, True])
def test_model_level_cuda_graph_steps_equal_eager_steps(do_sample):
    """The graph-replayed step runs the same kernels on the same buffers as the
    eager step: identical tokens, greedy or seeded sampling, EOS handling included."""
    model = _tiny_qwen2()
    torch.manual_seed(11)
    ids = torch.randint(0, 96, (6, 17), device=DEV)
    kw = dict(max_new_tokens=12, do_sample=do_sample, temperature=0.9, top_p=0.9, seed=1234,
              pad_token_id=0, eos_token_id=7)
    eager = pkg.paged_kv_decode(model, ids, torch.ones_like(ids), use_cuda_graph=False, **kw)
    graph = pkg.paged_kv_decode(model, ids, torch.ones_like(ids), use_cuda_graph=True, **kw)
    assert torch.equal(eager, graph)


def test_model_level_rows_do_not_share_pages():
    """Each row owns its pages (defect D1): a batched greedy rollout of different
    prompts equals each prompt rolled out alone. With one block table shared by
    all rows, as in the reference model path, rows overwrite each other's KV."""
    model = _tiny_qwen2(1)
    torch.manual_seed(8)
    ids = torch.randint(0, 96, (4, 13), device=DEV)
    batched = pkg.paged_kv_decode(model, ids, torch.ones_like(ids), max_new_tokens=8, do_sample=False)
    for i in range(4):
        single = pkg.paged_kv_decode(model, ids[i:i + 1], torch.ones_like(ids[i:i + 1]), max_new_tokens=8,
                                     do_sample=False)
        ref, gaps = _dense_rollout(model, ids[i:i + 1], 8)
        for got in (batched[i], single[0]):
            diff = (got != ref[0]).nonzero()
            if len(diff):
                assert float(gaps[0, int(diff[0])]) < 0.05


def _assert_matches_dense(got_row, ref_row, gap_row):
    diff = (got_row != ref_row).nonzero()
    if len(diff):  # only a near-tie in the dense logits may flip a greedy token
        first = int(diff[0])
        assert float(gap_row[first]) < 0.05, (first, float(gap_row[first]))


def test_model_level_group_shares_prompt_pages():
    """A GRPO group -- one prompt expanded to the micro-batch, as the trainer passes
    it -- is prefilled once with its full prompt pages shared: greedy rows are
    identical and match the dense rollout of the prompt alone."""
    model = _tiny_qwen2(2)
    torch.manual_seed(9)
    prompt = torch.randint(0, 96, (1, 37), device=DEV)  # 36 prefilled tokens: 2 shared pages + a tail of 4
    ids = prompt.expand(6, -1)
    got = pkg.paged_kv_decode(model, ids, torch.ones_like(prompt).expand(6, -1), max_new_tokens=10,
                              do_sample=False)
    assert got.shape == (6, 10) and (got == got[0]).all()
    ref, gaps = _dense_rollout(model, prompt, 10)
    _assert_matches_dense(got[0], ref[0], gaps[0])


@pytest.mark.parametrize("prompt_len", [33, 40])  # prefix on a page boundary / with a partial page
def test_model_level_interleaved_groups(prompt_len):
    model = _tiny_qwen2(3)
    torch.manual_seed(10)
    prompts = torch.randint(0, 96, (2, prompt_len), device=DEV)
    order = [0, 1, 1, 0, 1]
    ids = prompts[order]
    got = pkg.paged_kv_decode(model, ids, torch.ones_like(ids), max_new_tokens=8, do_sample=False)
    for g in range(2):
        ref, gaps = _dense_rollout(model, prompts[g:g + 1], 8)
        for row in (r for r, o in enumerate(order) if o == g):
            _assert_matches_dense(got[row], ref[0], gaps[0])
    unshared = pkg.paged_kv_decode(model, ids, torch.ones_like(ids), max_new_tokens=8, do_sample=False,
                                   share_prompt_pages=False)
    for g in range(2):
        ref, gaps = _dense_rollout(model, prompts[g:g + 1], 8)
        for row in (r for r, o in enumerate(order) if o == g):
            _assert_matches_dense(unshared[row], ref[0], gaps[0])


def test_model_level_group_rows_sample_independently():
    model = _tiny_qwen2(2)
    torch.manual_seed(12)
    prompt = torch.randint(0, 96, (1, 25), device=DEV)
    kw = dict(max_new_tokens=12, do_sample=True, temperature=1.0, top_p=0.95, seed=77, pad_token_id=0)
    a = pkg.paged_kv_decode(model, prompt.expand(8, -1), torch.ones_like(prompt).expand(8, -1), **kw)
    b = pkg.paged_kv_decode(model, prompt.expand(8, -1), torch.ones_like(prompt).expand(8, -1), **kw)
    assert torch.equal(a, b)  # seeded
    assert len({tuple(r.tolist()) for r in a}) > 1  # shared prompt pages, private draws


def test_facade_return_prompt_gives_generate_layout():
    model = _tiny_qwen2()
    torch.manual_seed(13)
    ids = torch.randint(1, 96, (3, 11), device=DEV)
    mask = torch.ones_like(ids)
    mask[1, :3] = 0  # left padding
    new = pkg.paged_kv_decode(model, ids, mask, max_new_tokens=5, do_sample=False)
    full = pkg.paged_kv_decode(model, ids, mask, max_new_tokens=5, do_sample=False, return_prompt=True)
    assert full.shape == (3, 16) and torch.equal(full[:, :11], ids)
    assert torch.equal(full[:, 11:], new.to(ids.dtype))  # the trainer's outputs[j, prompt_len:]


def test_model_level_wrapped_projections_take_the_module_path():
    """Projections that are not plain nn.Linear (a LoRA-wrapped layer in the trainer)
    are called as modules: no weight stacks, RoPE as its own launch. Same weights,
    same greedy tokens as the dense rollout."""

    class Wrapped(torch.nn.Linear):  # stands in for an adapter-wrapped projection
        pass

    model = _tiny_qwen2(4)
    for layer in model.model.layers:
        for owner, names in ((layer.self_attn, ("q_proj", "k_proj", "v_proj", "o_proj")),
                             (layer.mlp, ("gate_proj", "up_proj", "down_proj"))):
            for n in names:
                old = getattr(owner, n)
                new = Wrapped(old.in_features, old.out_features, bias=old.bias is not None,
                              device=old.weight.device, dtype=old.weight.dtype)
                new.load_state_dict(old.state_dict())
                setattr(owner, n, new)
    torch.manual_seed(14)
    ids = torch.randint(0, 96, (3, 19), device=DEV)
    got = pkg.paged_kv_decode(model, ids, torch.ones_like(ids), max_new_tokens=8, do_sample=False)
    for row in range(3):
        ref, gaps = _dense_rollout(model, ids[row:row + 1], 8)
        _assert_matches_dense(got[row], ref[0], gaps[0])
