"""Decode-step element-wise kernels (C ABI pkv_add_rmsnorm / pkv_silu_mul /
pkv_rope_qk) against the HF modules they replace in the rollout step:
Qwen2RMSNorm (with the residual add in front, as in a decoder layer), the SiLU
gate of Qwen2MLP, and apply_rotary_pos_emb."""

from __future__ import annotations

import pytest
import torch

from grpo_training_engine_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("hidden", [1536, 3584, 896, 4096, 104])
@pytest.mark.parametrize("with_residual", [False, True])
def test_add_rmsnorm_matches_qwen2_rmsnorm(hidden, with_residual):
    from transformers.models.qwen2.modeling_qwen2 import Qwen2RMSNorm

    g = torch.Generator(device=DEV).manual_seed(hidden)
    x = (torch.randn(96, hidden, device=DEV, generator=g) * 3).to(torch.bfloat16)
    r = (torch.randn(96, hidden, device=DEV, generator=g) * 5).to(torch.bfloat16)
    norm = Qwen2RMSNorm(hidden, eps=1e-6).to(DEV, torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(hidden, device=DEV, generator=g))
        s_ref = (r + x) if with_residual else x
        ref = norm(s_ref)
    out, total = ops.add_rmsnorm(x, norm.weight, norm.variance_epsilon, residual=r if with_residual else None)
    if with_residual:
        assert torch.equal(total, s_ref)  # the residual sum is bit-exact
    # fp32 statistics summed in another order: at most one bf16 step apart, rarely
    diff = (out.float() - ref.float()).abs()
    step = ref.float().abs() * 2.0 ** -7 + 1e-30
    assert bool((diff <= step).all())
    assert float((out != ref).float().mean()) < 0.01


@pytest.mark.parametrize("hq,hkv,d", [(12, 2, 128), (28, 4, 128), (4, 2, 64)])
def test_rope_qk_matches_apply_rotary_pos_emb(hq, hkv, d):
    from transformers import Qwen2Config
    from transformers.models.qwen2.modeling_qwen2 import Qwen2RotaryEmbedding, apply_rotary_pos_emb

    g = torch.Generator(device=DEV).manual_seed(d + hq)
    b = 37
    q = (torch.randn(b, hq * d, device=DEV, generator=g) * 2).to(torch.bfloat16)
    k = (torch.randn(b, hkv * d, device=DEV, generator=g) * 2).to(torch.bfloat16)
    cfg = Qwen2Config(hidden_size=hq * d, num_attention_heads=hq, num_key_value_heads=hkv, rope_theta=10000.0,
                      max_position_embeddings=40000)
    rot = Qwen2RotaryEmbedding(cfg).to(DEV)
    pos = torch.randint(0, 32768, (b, 1), device=DEV, generator=g)
    cos, sin = rot(q.view(b, 1, -1), pos)
    q_ref, k_ref = apply_rotary_pos_emb(q.view(b, 1, hq, d).transpose(1, 2), k.view(b, 1, hkv, d).transpose(1, 2),
                                        cos, sin)
    qo, ko = ops.rope_qk(q, k, cos.reshape(b, d), sin.reshape(b, d), hq, hkv, d)
    assert torch.equal(qo, q_ref[:, :, 0, :])
    assert torch.equal(ko, k_ref[:, :, 0, :])
    # q / k / v as column slices of one stacked projection, keys rotated in place
    qkv = torch.cat([q, k, k.flip(0)], dim=1)
    qs, ks = qkv[:, :hq * d], qkv[:, hq * d:(hq + hkv) * d]
    qo2, ko2 = ops.rope_qk(qs, ks, cos.reshape(b, d), sin.reshape(b, d), hq, hkv, d, k_out=ks)
    assert torch.equal(qo2, qo) and torch.equal(ko2, ko)
    assert ko2.data_ptr() == ks.data_ptr() and ko2.stride() == (qkv.stride(0), d, 1)
    assert torch.equal(qkv[:, :hq * d], q) and torch.equal(qkv[:, (hq + hkv) * d:], k.flip(0))


def test_silu_mul_matches_qwen2_mlp_gate():
    g = torch.Generator(device=DEV).manual_seed(1)
    gate = (torch.randn(128, 8960, device=DEV, generator=g) * 3).to(torch.bfloat16)
    up = (torch.randn(128, 8960, device=DEV, generator=g) * 3).to(torch.bfloat16)
    ref = torch.nn.functional.silu(gate) * up
    out = ops.silu_mul(gate, up)
    diff = (out.float() - ref.float()).abs()
    assert bool((diff <= ref.float().abs() * 2.0 ** -7 + 1e-30).all())
    assert float((out != ref).float().mean()) < 0.01


def test_glue_rejects_unaligned_rows():
    x = torch.randn(4, 100, device=DEV).to(torch.bfloat16)  # 200-byte rows
    with pytest.raises(RuntimeError):
        ops.add_rmsnorm(x, torch.ones(100, device=DEV, dtype=torch.bfloat16), 1e-6)


@pytest.mark.parametrize("name", ["rmsnorm_1536", "rmsnorm_3584", "rmsnorm_104"])
def test_add_rmsnorm_matches_the_reference_rmsnorm_kernel(name):
    """pkv_add_rmsnorm without a residual against the reference's fused_rmsnorm
    (src/triton_kernels/fused_ops.py:34-77, the norm its rollout step calls,
    paged_kv.py:706-710): the fixture (the reference kernel run by
    tests/golden/make_golden.py) is reproduced bit for bit by oracle.rmsnorm with
    the interpreter's truncating cast; with the GPU's nearest-even cast the
    oracle is the reference's arithmetic, and the kernel must match it except
    where the sum of squares, accumulated in another order, moves a product
    across a rounding boundary (at most one bf16 step, on few elements)."""
    import cases
    from conftest import load_golden
    from oracle import oracle

    case = next(c for c in cases.RMSNORM_CASES if c["name"] == name)
    ref_bits, _ = load_golden(name)
    inp = cases.make_rmsnorm_inputs(case)
    x = torch.from_numpy(inp["x"]).to(torch.bfloat16)
    w = torch.from_numpy(inp["weight"]).to(torch.bfloat16)
    assert torch.equal(oracle.rmsnorm(x, w, case["eps"], cast_rounding="rtz"),
                       torch.from_numpy(ref_bits).view(torch.bfloat16))
    want = oracle.rmsnorm(x, w, case["eps"])
    out, _ = ops.add_rmsnorm(x.to(DEV), w.to(DEV), case["eps"])
    out = out.cpu()
    diff = (out.float() - want.float()).abs()
    assert bool((diff <= want.float().abs() * 2.0 ** -7 + 1e-30).all())
    assert float((out != want).float().mean()) < 0.01
