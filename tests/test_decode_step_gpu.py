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


@pytest.mark.parametrize("preset,context,budget", [("popkv-q", 2048, 256), ("popkv-s", 3000, 700),
                                                   ("popkv-normal", 777, 1000)])
def test_graph_step_matches_oracle(cuda_device, preset, context, budget):
    tg, g = P.POPKV_PRESETS[preset]
    x = decode_inputs(context=context, seed=11, dtype="bf16")
    dev = cuda_device
    to = lambda a: torch.from_numpy(a).to(torch.bfloat16).to(dev)  # noqa: E731
    keys, values = to(x.keys[0]), to(x.values[0])
    cache = P.build_popkv_cache(keys, group_size=tg, dim_group_size=g, reserve_tokens=8)
    mapping = torch.from_numpy(head_to_kv(32, 8)).to(dev)
    step = SparseAttentionStep(cache, keys, values, mapping, budget=budget)
    q_host = to(x.queries).cpu().pin_memory()
    k_host = to(x.current_keys[0]).cpu().pin_memory()
    v_host = to(x.current_values[0]).cpu().pin_memory()
    out = step(q_host, k_host, v_host).clone()
    again = step(q_host, k_host, v_host).clone()
    assert torch.equal(out, again)
    eager = P.popkv_attention(to(x.queries[0]), keys, values, to(x.current_keys[0]),
                              to(x.current_values[0]), cache, mapping, budget=budget)
    torch.testing.assert_close(out[0], eager, atol=0, rtol=0)

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
