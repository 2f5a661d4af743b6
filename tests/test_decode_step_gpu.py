"""The graph-captured decode step (popkv_b200.decode) against the oracle and the eager path."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from popkv_b200 import popkv as P
from popkv_b200.decode import SparseAttentionStep
from popkv_b200.workloads import decode_inputs, head_to_kv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("host_io", [False, True])
@pytest.mark.parametrize("select", ["hist", "radix"])
@pytest.mark.parametrize("preset,context,budget", [("popkv-q", 2048, 256), ("popkv-s", 3000, 700),
                                                   ("popkv-normal", 777, 1000),
                                                   ("popkv-q", 32768, 4096)])  # the benchmark's step
def test_graph_step_matches_oracle(cuda_device, preset, context, budget, select, host_io):
    tg, g = P.POPKV_PRESETS[preset]
    x = decode_inputs(context=context, seed=11, dtype="bf16")
    dev = cuda_device
    to = lambda a: torch.from_numpy(a).to(torch.bfloat16).to(dev)  # noqa: E731
    keys, values = to(x.keys[0]), to(x.values[0])
    cache = P.build_popkv_cache(keys, group_size=tg, dim_group_size=g, reserve_tokens=8)
    mapping = torch.from_numpy(head_to_kv(32, 8)).to(dev)
    step = SparseAttentionStep(cache, keys, values, mapping, budget=budget, select=select, host_io=host_io)
    assert step.select == select
    q_host = to(x.queries).cpu().pin_memory()
    k_host = to(x.current_keys[0]).cpu().pin_memory()
    v_host = to(x.current_values[0]).cpu().pin_memory()
    out = step(q_host, k_host, v_host)
    torch.cuda.current_stream(dev).synchronize()  # host_io: the result lands in pinned host memory
    out = out.clone()
    again = step(q_host, k_host, v_host)
    torch.cuda.current_stream(dev).synchronize()
    assert torch.equal(out, again.clone())
    out = out.to(dev)
    eager = P.popkv_attention(to(x.queries[0]), keys, values, to(x.current_keys[0]),
                              to(x.current_values[0]), cache, mapping, budget=budget)
    # The graph's attention kernels sum in another order than the eager chain:
    # equal up to bf16 output rounding.
    assert (out[0].float() - eager.float()).abs().max().item() <= 2 ** -6

    kbits, qbits = x.bits("keys")[0], x.bits("queries")
    opk = oracle.pack(kbits, "bf16", token_group_size=tg, dim_group_size=g)
    enc = oracle.query_encode(qbits, "bf16", dim_group_size=g)
    _, s16 = oracle.score(enc, opk, head_to_kv=head_to_kv(32, 8), tokens=context,
                          dim_group_size=g, head_dim=128)
    idx = oracle.select_with_current(s16, budget, context)[0]
    np.testing.assert_array_equal(step.indices[0].cpu().numpy(), idx)
    want = oracle.attention(qbits[0], "bf16", kbits, x.bits("values")[0], "bf16",
                            x.bits("current_keys")[0], x.bits("current_values")[0], idx,
                            head_to_kv(32, 8))
    err = np.abs(out[0].float().cpu().numpy() - want)
    assert err.max() <= 2e-2 and err.mean() <= 2e-3


@pytest.mark.parametrize("preset,context,budget", [("popkv-q", 32768, 4096), ("popkv-s", 5000, 512),
                                                   ("popkv-normal", 1000, 2000), ("popkv-q", 300, 64)])
def test_fused_retrieve_matches_unfused_and_oracle(cuda_device, preset, context, budget):
    """popkv_retrieve == score -> topk -> split attention (scores and indices bit-exact)."""
    tg, g = P.POPKV_PRESETS[preset]
    x = decode_inputs(context=context, seed=5, dtype="bf16")
    dev = cuda_device
    to = lambda a: torch.from_numpy(a).to(torch.bfloat16).to(dev)  # noqa: E731
    keys, values = to(x.keys[0]), to(x.values[0])
    cache = P.build_popkv_cache(keys, group_size=tg, dim_group_size=g, reserve_tokens=8)
    mapping = torch.from_numpy(head_to_kv(32, 8)).to(dev)
    q = to(x.queries)
    ck, cv = to(x.current_keys[0]), to(x.current_values[0])
    out, scores, indices = P.popkv_retrieve(q, cache.packed, keys, values, ck, cv, mapping,
                                            tokens=context, budget=budget, dim_group_size=g,
                                            return_scores=True, return_indices=True)
    from popkv_b200 import popkv_cuda as C
    want_scores = C.score(q, cache.packed, head_to_kv=mapping, tokens=context, dim_group_size=g)
    assert torch.equal(scores, want_scores)
    want_idx = P.select_tokens(want_scores, budget=budget, prefix_tokens=context)
    assert torch.equal(indices, want_idx)
    eager = P.popkv_attention(q[0], keys, values, ck, cv, cache, mapping, budget=budget)
    err = (out[0].float() - eager.float()).abs()
    assert err.max().item() <= 2 ** -6
    kbits, qbits = x.bits("keys")[0], x.bits("queries")
    opk = oracle.pack(kbits, "bf16", token_group_size=tg, dim_group_size=g)
    enc = oracle.query_encode(qbits, "bf16", dim_group_size=g)
    _, s16 = oracle.score(enc, opk, head_to_kv=head_to_kv(32, 8), tokens=context,
                          dim_group_size=g, head_dim=128)
    idx = oracle.select_with_current(s16, budget, context)[0]
    np.testing.assert_array_equal(indices[0].cpu().numpy(), idx)
    want = oracle.attention(qbits[0], "bf16", kbits, x.bits("values")[0], "bf16",
                            x.bits("current_keys")[0], x.bits("current_values")[0], idx,
                            head_to_kv(32, 8))
    e = np.abs(out[0].float().cpu().numpy() - want)
    assert e.max() <= 2e-2 and e.mean() <= 2e-3


def test_fused_retrieve_zero_context(cuda_device):
    """With no cached token the output is the current value (the only slot)."""
    dev = cuda_device
    keys = torch.zeros(8, 0, 128, dtype=torch.bfloat16, device=dev)
    cache_keys = torch.randn(8, 64, 128, device=dev).to(torch.bfloat16)
    cache = P.build_popkv_cache(cache_keys, group_size=64, dim_group_size=64, reserve_tokens=0)
    q = torch.randn(1, 32, 128, device=dev).to(torch.bfloat16)
    ck = torch.randn(8, 128, device=dev).to(torch.bfloat16)
    cv = torch.randn(8, 128, device=dev).to(torch.bfloat16)
    mapping = torch.from_numpy(head_to_kv(32, 8)).to(dev)
    out = P.popkv_retrieve(q, cache.packed, cache_keys, cache_keys, ck, cv, mapping, tokens=0,
                           budget=16, dim_group_size=64)
    torch.testing.assert_close(out[0].float(), cv[mapping].float(), atol=0, rtol=0)


@pytest.mark.parametrize("chunks", [2, 4, 8])
@pytest.mark.parametrize("select", ["radix", "hist"])
def test_chunked_step_equals_unchunked(cuda_device, chunks, select):
    """KV-head chunks on forked streams compute exactly what the single chain computes."""
    x = decode_inputs(context=5000, seed=3, dtype="bf16")
    dev = cuda_device
    to = lambda a: torch.from_numpy(a).to(torch.bfloat16).to(dev)  # noqa: E731
    keys, values = to(x.keys[0]), to(x.values[0])
    tg, g = P.POPKV_PRESETS["popkv-q"]
    cache = P.build_popkv_cache(keys, group_size=tg, dim_group_size=g, reserve_tokens=8)
    mapping = torch.from_numpy(head_to_kv(32, 8)).to(dev)
    q, ck, cv = to(x.queries), to(x.current_keys[0]), to(x.current_values[0])
    one = SparseAttentionStep(cache, keys, values, mapping, budget=700, select=select)
    want = one(q, ck, cv).clone()
    many = SparseAttentionStep(cache, keys, values, mapping, budget=700, select=select, chunks=chunks)
    for _ in range(2):
        got = many(q, ck, cv).clone()
        torch.cuda.synchronize()
        assert torch.equal(many.indices, one.indices)
        assert torch.equal(got, want)
    eager = many.run_eager().clone()
    assert torch.equal(eager, want)


def test_chunked_step_rejects_unsupported(cuda_device):
    dev = cuda_device
    keys = torch.randn(8, 512, 128, device=dev).to(torch.bfloat16)
    cache = P.build_popkv_cache(keys, group_size=64, dim_group_size=64, reserve_tokens=0)
    mapping = torch.from_numpy(head_to_kv(32, 8)).to(dev)
    with pytest.raises(ValueError, match="divide"):
        SparseAttentionStep(cache, keys, keys, mapping, budget=64, chunks=3, use_graph=False)
    with pytest.raises(ValueError, match="consecutive"):
        SparseAttentionStep(cache, keys, keys, mapping.flip(0), budget=64, chunks=2, use_graph=False)


def test_host_io_step_moves_inputs_and_output_in_the_graph(cuda_device):
    """host_io: the captured graph copies q | k | v in and the output out."""
    x = decode_inputs(context=3000, seed=21, dtype="bf16")
    dev = cuda_device
    to = lambda a: torch.from_numpy(a).to(torch.bfloat16)  # noqa: E731
    keys, values = to(x.keys[0]).to(dev), to(x.values[0]).to(dev)
    tg, g = P.POPKV_PRESETS["popkv-s"]
    cache = P.build_popkv_cache(keys, group_size=tg, dim_group_size=g, reserve_tokens=8)
    mapping = torch.from_numpy(head_to_kv(32, 8)).to(dev)
    plain = SparseAttentionStep(cache, keys, values, mapping, budget=500)
    want = plain(to(x.queries).to(dev), to(x.current_keys[0]).to(dev), to(x.current_values[0]).to(dev)).clone()
    step = SparseAttentionStep(cache, keys, values, mapping, budget=500, host_io=True)
    assert step.host_queries.is_pinned() and step.host_output.is_pinned()
    for _ in range(2):
        out = step(to(x.queries), to(x.current_keys[0]), to(x.current_values[0]))
        torch.cuda.synchronize()
        assert out.data_ptr() == step.host_output.data_ptr()
        assert torch.equal(out, want.cpu())
    # Writing the staging views directly, then calling with them, skips the host copy.
    step.host_queries.copy_(to(x.queries))
    out = step(step.host_queries, step.host_current_keys, step.host_current_values)
    torch.cuda.synchronize()
    assert torch.equal(out, want.cpu())
    # Device inputs bypass the staging buffers and return the device output.
    dev_out = step(to(x.queries).to(dev), to(x.current_keys[0]).to(dev), to(x.current_values[0]).to(dev))
    assert dev_out.is_cuda and torch.equal(dev_out, want)


@pytest.mark.parametrize("preset,budget,host_io", [("popkv-q", 512, False), ("popkv-s", 300, True)])
def test_device_length_step_serves_every_length(cuda_device, preset, budget, host_io):
    """One captured step with the cache length on the device, replayed across appended
    tokens, equals a fresh step captured at each length (bit for bit)."""
    dev = cuda_device
    tg, g = P.POPKV_PRESETS[preset]
    gen = torch.Generator().manual_seed(budget)
    kvh, qh, t0, cap = 8, 32, 1000 - tg // 2, 1200
    keys = torch.randn(kvh, cap, 128, generator=gen).to(torch.bfloat16).to(dev)
    values = torch.randn(kvh, cap, 128, generator=gen).to(torch.bfloat16).to(dev)
    cache = P.build_popkv_cache(keys[:, :t0].contiguous(), group_size=tg, dim_group_size=g,
                                reserve_tokens=cap - t0)
    mapping = torch.from_numpy(head_to_kv(qh, kvh)).to(dev)
    dyn = SparseAttentionStep(cache, keys, values, mapping, budget=budget, max_tokens=cap - 1, host_io=host_io)
    for _ in range(tg + 3):  # crosses a token-group boundary
        t = cache.token_count
        q = torch.randn(1, qh, 128, generator=gen).to(torch.bfloat16).to(dev)
        ck = torch.randn(kvh, 128, generator=gen).to(torch.bfloat16).to(dev)
        cv = torch.randn(kvh, 128, generator=gen).to(torch.bfloat16).to(dev)
        static = SparseAttentionStep(cache, keys[:, :t], values[:, :t], mapping, budget=budget)
        want = static(q, ck, cv).clone()
        dyn.set_length()
        if host_io:
            dyn.host_queries.copy_(q.cpu().view_as(dyn.host_queries))
            dyn.host_current_keys.copy_(ck.cpu().view_as(dyn.host_current_keys))
            dyn.host_current_values.copy_(cv.cpu().view_as(dyn.host_current_values))
            got = dyn(dyn.host_queries, dyn.host_current_keys, dyn.host_current_values)
            torch.cuda.current_stream().synchronize()
            got = got.to(dev)
        else:
            got = dyn(q, ck, cv).clone()
        assert torch.equal(got.view_as(want), want), f"length {t}"
        P.append_popkv_kv(cache, keys, values, ck, cv)
    with pytest.raises(ValueError, match="max_tokens"):
        SparseAttentionStep(cache, keys, values, mapping, budget=budget, max_tokens=cap + 1)
