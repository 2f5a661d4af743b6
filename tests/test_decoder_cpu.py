"""Host-side pieces of the full-model decode, checked on CPU.

The eager helpers (rotary tables, RoPE, RMSNorm) define the rounding points the
decode kernels follow; here they are pinned to transformers' Llama modules,
which the reference decoder calls (popkv.py:974-987, :1011-1016, :1109).
"""
from __future__ import annotations

import pytest
import torch

from popkv_b200.decoder import (DECODE_METHODS, LLAMA31_8B, LlamaConfig, LlamaWeights, apply_rope, rms_norm,
                                rope_tables)

transformers = pytest.importorskip("transformers")
from transformers.models.llama import modeling_llama as ml  # noqa: E402


def _hf_config():
    return transformers.LlamaConfig(hidden_size=256, intermediate_size=512, num_attention_heads=2,
                                    num_key_value_heads=1, head_dim=128, num_hidden_layers=1, vocab_size=64,
                                    rope_theta=500000.0, rms_norm_eps=1e-5, max_position_embeddings=8192)


def test_rope_tables_match_transformers_rotary_embedding():
    cfg = LlamaConfig(hidden_size=256, num_attention_heads=2, num_key_value_heads=1, intermediate_size=512,
                      vocab_size=64, num_hidden_layers=1)
    rot = ml.LlamaRotaryEmbedding(config=_hf_config())
    positions = torch.arange(0, 5000)[None]
    x = torch.zeros(1, 1, 128, dtype=torch.bfloat16)
    cos_hf, sin_hf = rot(x, positions)
    cos, sin = rope_tables(cfg, 5000, "cpu")
    assert torch.equal(cos_hf[0, :, :64], cos) and torch.equal(cos_hf[0, :, 64:], cos)
    assert torch.equal(sin_hf[0, :, :64], sin) and torch.equal(sin_hf[0, :, 64:], sin)


def test_apply_rope_matches_transformers():
    gen = torch.Generator().manual_seed(0)
    q = torch.randn(1, 4, 7, 128, generator=gen).to(torch.bfloat16)
    k = torch.randn(1, 2, 7, 128, generator=gen).to(torch.bfloat16)
    cfg = LlamaConfig(hidden_size=256, num_attention_heads=2, num_key_value_heads=1, intermediate_size=512,
                      vocab_size=64, num_hidden_layers=1)
    cos, sin = rope_tables(cfg, 7, "cpu")
    cos2, sin2 = torch.cat([cos, cos], -1)[None], torch.cat([sin, sin], -1)[None]
    rq, rk = ml.apply_rotary_pos_emb(q, k, cos2, sin2)
    assert torch.equal(apply_rope(q, cos, sin), rq)
    assert torch.equal(apply_rope(k, cos, sin), rk)


def test_rms_norm_matches_transformers():
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(3, 256, generator=gen).to(torch.bfloat16)
    norm = ml.LlamaRMSNorm(256, eps=1e-5)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(256, generator=gen))
    norm = norm.to(torch.bfloat16)
    assert torch.equal(rms_norm(x, norm.weight, 1e-5), norm(x))


def test_config_validation_and_defaults():
    assert LLAMA31_8B.hidden_size == 4096 and LLAMA31_8B.intermediate_size == 14336
    assert LLAMA31_8B.vocab_size == 128256 and LLAMA31_8B.rope_theta == 500000.0
    assert set(DECODE_METHODS) == {"full", "popkv-q", "popkv-s", "popkv-normal"}
    with pytest.raises(ValueError, match="head_dim"):
        LlamaConfig(head_dim=64).validate()
    with pytest.raises(ValueError, match="4 query heads"):
        LlamaConfig(num_attention_heads=64, num_key_value_heads=8).validate()


def test_weights_from_module_fuse_projections():
    model = transformers.LlamaForCausalLM(_hf_config())
    w = LlamaWeights.from_module(model, device="cpu")
    layer = model.model.layers[0]
    a, m = layer.self_attn, layer.mlp
    assert w.layers[0].qkv.shape == (128 * 4, 256)
    assert torch.equal(w.layers[0].qkv[:256], a.q_proj.weight.to(torch.bfloat16))
    assert torch.equal(w.layers[0].qkv[256:384], a.k_proj.weight.to(torch.bfloat16))
    assert torch.equal(w.layers[0].gate_up[512:], m.up_proj.weight.to(torch.bfloat16))
    assert w.config.rope_theta == 500000.0
    # Bytes a batch-1 decode step streams: every matrix but the embedding.
    per_layer = (512 * 256 + 256 * 256 + 2 * 512 * 256 + 256 * 512 + 2 * 256) * 2
    assert w.bytes_per_token() == per_layer + (64 * 256 + 256) * 2


def test_kv_head_shard_takes_its_heads_qkv_rows():
    """A world-N decoder keeps rank r's query heads and KV heads of the fused q|k|v projection."""
    from popkv_b200.decoder import LlamaSparseDecoder
    cfg = LlamaConfig(hidden_size=1024, num_attention_heads=8, num_key_value_heads=4, intermediate_size=512,
                      vocab_size=64, num_hidden_layers=1)
    w = LlamaWeights.random(cfg, device="cpu", seed=3)
    full = w.layers[0].qkv.view(8 + 2 * 4, 128, 1024)
    world = 2
    for rank in range(world):
        dec = LlamaSparseDecoder(w, method="full", max_context=16, rank=rank, world=world, use_graph=False)
        assert dec.qh == 4 and dec.kvh == 2
        local = dec.qkv_weights[0].view(4 + 2 * 2, 128, 1024)
        q_heads = range(4 * rank, 4 * rank + 4)
        kv_heads = range(2 * rank, 2 * rank + 2)
        want = torch.cat([full[list(q_heads)], full[[8 + h for h in kv_heads]], full[[12 + h for h in kv_heads]]])
        assert torch.equal(local, want)
        assert tuple(dec.k_cache[0].shape) == (1, 2, 16, 128)
    with pytest.raises(ValueError, match="divide"):
        LlamaSparseDecoder(w, method="full", max_context=16, rank=0, world=3, use_graph=False)
