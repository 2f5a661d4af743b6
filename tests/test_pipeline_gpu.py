"""End-to-end decode step at the benchmark configurations, checked against the oracle.

Config 0 (fp32, T=4096, budget 512, PopKV-S) and config 1 (bf16, T=32768,
budget 4096, PopKV-Q) of the benchmark, on the seeded synthetic inputs of
popkv_b200.workloads.  Top-k indices are compared bit for bit (they depend on
bit-exact scores); the attention output within max-abs 2e-2 / mean-abs 2e-3 of
the float64 oracle over the same indices.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from popkv_b200 import popkv as P
from popkv_b200 import popkv_cuda as C
from popkv_b200 import sparse_kernels as S
from popkv_b200.workloads import decode_inputs, head_to_kv
from tests.helpers import bits, planes_to_numpy, random_keys, to_oracle

pytestmark = pytest.mark.gpu

CONFIGS = {
    "config0_popkv_s_fp32_4k": dict(context=4096, budget=512, preset="popkv-s", dtype="f32"),
    "config1_popkv_q_bf16_32k": dict(context=32768, budget=4096, preset="popkv-q", dtype="bf16"),
}


@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_decode_step_matches_oracle(cuda_device, name):
    cfg = CONFIGS[name]
    tg, g = P.POPKV_PRESETS[cfg["preset"]]
    x = decode_inputs(context=cfg["context"], dtype=cfg["dtype"], seed=0)
    tdtype = torch.float32 if cfg["dtype"] == "f32" else torch.bfloat16
    dev = cuda_device
    keys = torch.from_numpy(x.keys[0]).to(tdtype).to(dev)
    values = torch.from_numpy(x.values[0]).to(tdtype).to(dev)
    queries = torch.from_numpy(x.queries[0]).to(tdtype).to(dev)
    cur_k = torch.from_numpy(x.current_keys[0]).to(tdtype).to(dev)
    cur_v = torch.from_numpy(x.current_values[0]).to(tdtype).to(dev)
    mapping = torch.from_numpy(head_to_kv(32, 8)).to(dev)
    T = cfg["context"]

    cache = P.build_popkv_cache(keys, group_size=tg, dim_group_size=g, reserve_tokens=256)
    enc = C.query_encode(queries.unsqueeze(0).contiguous(), dim_group_size=g)
    scores = C.score_encoded(enc, cache.packed, head_to_kv=mapping, tokens=cache.token_count,
                             dim_group_size=g)
    indices = P.select_tokens(scores, budget=cfg["budget"], prefix_tokens=T)[0]
    out = P.popkv_attention(queries, keys, values, cur_k, cur_v, cache, mapping, budget=cfg["budget"])

    # Oracle chain on the same inputs.
    karr, ktag = to_oracle(keys)
    opk = oracle.pack(karr, ktag, token_group_size=tg, dim_group_size=g)
    gpk = planes_to_numpy(cache.packed)
    for a, b in zip(gpk, opk):
        np.testing.assert_array_equal(a[:, :T], b[:, :T])
    qarr, qtag = to_oracle(queries.unsqueeze(0))
    oenc = oracle.query_encode(qarr, qtag, dim_group_size=g)
    for a, b in zip(enc, oenc):
        np.testing.assert_array_equal(a.cpu().numpy(), b)
    _, s16 = oracle.score(oenc, opk, head_to_kv=head_to_kv(32, 8), tokens=T, dim_group_size=g,
                          head_dim=128)
    np.testing.assert_array_equal(bits(scores), s16)
    oidx = oracle.select_with_current(s16, cfg["budget"], T)[0]
    np.testing.assert_array_equal(indices.cpu().numpy(), oidx)

    varr, _ = to_oracle(values)
    ck, _ = to_oracle(cur_k)
    cv, _ = to_oracle(cur_v)
    want = oracle.attention(qarr[0], qtag, karr, varr, ktag, ck, cv, oidx, head_to_kv(32, 8))
    err = np.abs(out.float().cpu().numpy().astype(np.float64) - want)
    # bf16 output rounding dominates for config 1; fp32 for config 0.
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, (err.max(), err.mean())

    # Size-independent properties at full size.
    assert indices.shape == (32, min(cfg["budget"] - 1, T) + 1)
    assert torch.all(indices[:, -1] == T)
    assert torch.all(indices[:, 1:-1] > indices[:, :-2])


def test_sparse_attention_full_size_reference_case(cuda_device):
    """tests/test_sparse_kernels.py:118-141 at full size: T=32768, budget 4096, masked slots."""
    gen = torch.Generator().manual_seed(104)
    dev = cuda_device
    q_heads, kv_heads, tokens, dim = 8, 2, 32768, 128
    queries = torch.randn(q_heads, dim, generator=gen).to(torch.bfloat16).to(dev)
    keys = torch.randn(kv_heads, tokens, dim, generator=gen).to(torch.bfloat16).to(dev)
    values = torch.randn(kv_heads, tokens, dim, generator=gen).to(torch.bfloat16).to(dev)
    cur_k = torch.randn(kv_heads, dim, generator=gen).to(torch.bfloat16).to(dev)
    cur_v = torch.randn(kv_heads, dim, generator=gen).to(torch.bfloat16).to(dev)
    mapping = torch.arange(q_heads, device=dev) // 4
    indices = torch.randint(tokens, (q_heads, 4096), generator=gen).to(dev)
    indices[:, -1] = tokens
    valid = torch.ones_like(indices, dtype=torch.bool)
    valid[:, -7:-1] = False
    out = S.indexed_attention_split(queries, keys, values, cur_k, cur_v, indices, mapping, valid,
                                    split_tokens=256)
    # Dense attention over the same indices (the reference test's materialized oracle).
    safe = indices.clamp_max(tokens - 1)
    kvh = mapping[:, None].expand_as(safe)
    sel_k = torch.where(indices.eq(tokens)[..., None], cur_k[mapping][:, None], keys[kvh, safe]).float()
    sel_v = torch.where(indices.eq(tokens)[..., None], cur_v[mapping][:, None], values[kvh, safe]).float()
    logits = (sel_k @ queries.float()[:, :, None])[..., 0] / np.sqrt(dim)
    logits = logits.masked_fill(~valid, float("-inf"))
    dense = (torch.softmax(logits, -1)[:, None] @ sel_v)[:, 0]
    err = (out.float() - dense).abs()
    assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3


@pytest.mark.parametrize("g,tg", [(16, 128), (64, 64), (32, 32)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_append_kv_from_static_cache_matches_prepack(cuda_device, g, tg, dtype):
    """popkv_append_kv (KV append fused with the re-encode) == prepack of all tokens, across a seal."""
    gen = torch.Generator().manual_seed(g + tg)
    kvh, t0, extra = 4, 3 * tg - 5, 9
    full_k = random_keys(gen, (kvh, t0 + extra, 128), dtype, cuda_device)
    full_v = torch.randn(kvh, t0 + extra, 128, generator=gen).to(dtype).to(cuda_device)
    key_cache = torch.zeros(kvh, t0 + extra + 7, 128, dtype=dtype, device=cuda_device)
    value_cache = torch.zeros_like(key_cache)
    key_cache[:, :t0] = full_k[:, :t0]
    value_cache[:, :t0] = full_v[:, :t0]
    cache = P.build_popkv_cache(full_k[:, :t0], group_size=tg, dim_group_size=g, reserve_tokens=extra + 7)
    for i in range(extra):
        P.append_popkv_kv(cache, key_cache, value_cache, full_k[:, t0 + i], full_v[:, t0 + i])
    torch.cuda.synchronize()
    n = t0 + extra
    assert cache.token_count == n and cache.sealed_tokens == (n // tg) * tg
    assert torch.equal(key_cache[:, :n], full_k) and torch.equal(value_cache[:, :n], full_v)
    want = C.pack_keys(full_k.contiguous(), token_group_size=tg, dim_group_size=g)
    for got, exp in zip(cache.packed, want):
        assert torch.equal(got[:, :n], exp[:, :n])
