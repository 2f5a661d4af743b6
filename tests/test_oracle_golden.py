"""Pin the CPU oracle to the reference's own outputs (tests/golden/popkv_golden.npz).

The fixture was produced by tests/golden/make_golden.py from the reference's
readable oracles and its Triton kernels; tolerances are the reference tests'
own (tests/test_popkv.py:200-211, :276-300, :334-352;
tests/test_sparse_kernels.py:118-141).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle

GROUPS = (16, 32, 64)
DIMS = (32, 64, 96, 127, 128)


def test_hand_computable_query(golden):
    q = golden["hand/q"].astype(np.float32)
    sign, mag, low, delta = oracle.query_encode(q, "f32", dim_group_size=32)
    assert int(sign.item()) == 0b10101 == int(golden["hand/sign"].item())
    assert int(mag.item()) == 0b01100 == int(golden["hand/mag"].item())
    np.testing.assert_allclose(low, golden["hand/low"], rtol=0, atol=1e-7)
    np.testing.assert_allclose(delta, golden["hand/delta"], rtol=0, atol=1e-6)
    assert float(low.item()) == np.float32(2.0) / np.float32(3.0)


@pytest.mark.parametrize("tag", ["pos", "neg"])
def test_empty_bucket_query(golden, tag):
    q = golden[f"empty_{tag}/q"].astype(np.float32)
    sign, mag, low, delta = oracle.query_encode(q, "f32", dim_group_size=32)
    np.testing.assert_array_equal(mag, golden[f"empty_{tag}/mag"])
    assert int(mag.item()) == -1
    np.testing.assert_array_equal(sign, golden[f"empty_{tag}/sign"])
    np.testing.assert_array_equal(low, golden[f"empty_{tag}/low"])
    np.testing.assert_array_equal(delta, golden[f"empty_{tag}/delta"])


@pytest.mark.parametrize("group", GROUPS)
@pytest.mark.parametrize("dim", DIMS)
def test_query_encode_matches_reference(golden, group, dim):
    tag = f"g{group}_d{dim}"
    out = oracle.query_encode(golden[f"qenc/{tag}/q"], "bf16", dim_group_size=group)
    np.testing.assert_array_equal(out[0], golden[f"qenc/{tag}/sign"])
    np.testing.assert_array_equal(out[1], golden[f"qenc/{tag}/mag"])
    np.testing.assert_allclose(out[2], golden[f"qenc/{tag}/low"], atol=2e-5, rtol=2e-5)
    np.testing.assert_allclose(out[3], golden[f"qenc/{tag}/delta"], atol=2e-5, rtol=2e-5)


def _check_key_encode(golden, prefix, packed):
    np.testing.assert_array_equal(packed[0], golden[f"{prefix}/sign"])
    np.testing.assert_array_equal(packed[1], golden[f"{prefix}/mag"])
    np.testing.assert_allclose(oracle.half_bits_to_float(packed[2]), golden[f"{prefix}/low"],
                               atol=2e-3, rtol=2e-3)
    np.testing.assert_allclose(oracle.half_bits_to_float(packed[3]), golden[f"{prefix}/delta"],
                               atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize("group", GROUPS)
@pytest.mark.parametrize("dim", DIMS)
def test_key_encode_and_scores_match_reference(golden, group, dim):
    tag = f"g{group}_d{dim}"
    keys = golden[f"kenc/{tag}/k"]
    packed = oracle.pack(keys, "bf16", token_group_size=32, dim_group_size=group)
    _check_key_encode(golden, f"kenc/{tag}", packed)
    enc = oracle.query_encode(golden[f"qenc/{tag}/q"], "bf16", dim_group_size=group)
    s32, s16 = oracle.score(enc, packed, head_to_kv=golden["mapping8"], tokens=37,
                            dim_group_size=group, head_dim=dim)
    actual = oracle.half_bits_to_float(s16) if dim == 128 else s32
    np.testing.assert_allclose(actual, golden[f"score/{tag}"], atol=0.15, rtol=0.025)


@pytest.mark.parametrize("group,tg", [(32, t) for t in (5, 8, 10, 16, 32, 64, 125, 128, 500)]
                         + [(16, t) for t in (8, 16, 32, 64, 128)]
                         + [(64, t) for t in (8, 16, 32, 64, 128)])
def test_token_groups_match_reference(golden, group, tg):
    prefix = f"tg/g{group}_tg{tg}"
    keys = golden[f"{prefix}/k"]
    packed = oracle.pack(keys, "bf16", token_group_size=tg, dim_group_size=group)
    _check_key_encode(golden, prefix, packed)
    enc = oracle.query_encode(golden[f"{prefix}/q"], "bf16", dim_group_size=group)
    _, s16 = oracle.score(enc, packed, head_to_kv=golden["mapping8"], tokens=keys.shape[1],
                          dim_group_size=group, head_dim=128)
    np.testing.assert_allclose(oracle.half_bits_to_float(s16), golden[f"{prefix}/score"],
                               atol=0.15, rtol=0.025)


@pytest.mark.parametrize("group,tg", [(16, 8), (32, 5), (32, 32), (64, 64), (16, 128)])
def test_incremental_append_crosses_group_boundaries(golden, group, tg):
    """Appending one token at a time re-encodes the active group (popkv.py:438-459).

    After every append the planes equal a fresh encode of all keys so far
    (tests/test_popkv.py:355-372 asserts the same against reference_key_encode).
    """
    keys = golden[f"tg/g{group}_tg{tg}/k"]
    total = keys.shape[1]
    start = tg - 1
    packed = oracle.pack(keys[:, :start], "bf16", token_group_size=tg, dim_group_size=group,
                         token_capacity=total)
    sealed = (start // tg) * tg
    for count in range(start + 1, total + 1):
        active = keys[:, sealed:count]
        oracle.pack(active, "bf16", token_group_size=tg, dim_group_size=group,
                    token_offset=sealed, out=packed)
        full = oracle.pack(keys[:, :count], "bf16", token_group_size=tg, dim_group_size=group)
        for mine, want in zip(packed, full):
            np.testing.assert_array_equal(mine[:, :count], want[:, :count])
        if active.shape[1] == tg:
            sealed += tg


@pytest.mark.parametrize("group", GROUPS)
def test_popcount_decomposition_matches_reconstruction(golden, group):
    q = golden["bitwise/q"].astype(np.float32)
    k = golden["bitwise/k"].astype(np.float32)
    enc = oracle.query_encode(q, "f32", dim_group_size=group)
    packed = oracle.pack(k, "f32", token_group_size=32, dim_group_size=group)
    s32, _ = oracle.score(enc, packed, head_to_kv=np.array([0]), tokens=k.shape[1],
                          dim_group_size=group, head_dim=q.shape[-1])
    np.testing.assert_allclose(golden[f"bitwise/g{group}"], golden[f"bitwise/direct_g{group}"],
                               atol=2e-6, rtol=2e-6)
    np.testing.assert_allclose(s32, golden[f"bitwise/g{group}"], atol=2e-5, rtol=2e-5)


def test_current_slot_reserved(golden):
    chosen = golden["append_current/in"]
    scores = np.zeros((2, 12), np.float32)
    for row, picks in enumerate(chosen):
        scores[row, picks] = 1.0
    out = oracle.select_with_current(scores, budget=3, prefix_tokens=11)
    np.testing.assert_array_equal(out, golden["append_current/out"])


@pytest.mark.parametrize("k", (1, 255, 511, 1024))
def test_topk_matches_torch_topk_modulo_ties(golden, k):
    """Same selection as torch.topk(sorted=False) up to the order of equal scores."""
    scores = golden["topk/scores16"]
    mine = oracle.topk(scores, k)
    want = golden[f"topk/k{k}"].astype(np.int64)
    values = oracle.half_bits_to_float(scores)
    for row in range(scores.shape[1]):
        v = values[0, row]
        kth = np.sort(v[want[0, row]])[0]
        assert np.sort(v[mine[0, row]])[0] == kth
        above_mine = set(mine[0, row][v[mine[0, row]] > kth])
        above_want = set(want[0, row][v[want[0, row]] > kth])
        assert above_mine == above_want
        assert np.all(np.diff(mine[0, row]) > 0)
        tied = np.flatnonzero(v == kth)
        taken = np.sort(mine[0, row][v[mine[0, row]] == kth])
        np.testing.assert_array_equal(taken, tied[:len(taken)])


def test_split_attention_matches_reference_triton(golden):
    prefix = int(golden["attn/prefix_tokens"])
    keys = golden["attn/k_store"][:, :prefix]
    values = golden["attn/v_store"][:, :prefix]
    partials = oracle.attn_partial(golden["attn/q"], "bf16", keys, values, "bf16",
                                   golden["attn/cur_k"], golden["attn/cur_v"],
                                   golden["attn/indices"], golden["attn/mapping"],
                                   golden["attn/valid"], split_tokens=256)
    ref = golden["attn/partials"]
    np.testing.assert_allclose(partials[..., 0], ref[..., 0], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(partials[..., 1], ref[..., 1], atol=1e-4, rtol=1e-5)
    np.testing.assert_allclose(partials[..., 2:], ref[..., 2:], atol=1e-4, rtol=1e-5)
    merged = oracle.attn_merge(partials)
    np.testing.assert_allclose(merged, golden["attn/merged"], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(merged, golden["attn/dense"], atol=1e-5, rtol=1e-5)


def test_float_to_half_rounding_edges():
    lib = oracle.lib()
    for value in (0.0, -0.0, 1.0, 65504.0, 65519.99, 65520.0, 2.0 ** -24, 2.0 ** -25,
                  3 * 2.0 ** -26, 6.1e-5, 1e-8, -3.14159, 0.1, 1 / 3):
        want = np.array(value, np.float32).astype(np.float16).view(np.uint16)
        assert lib.oracle_float_to_half(float(np.float32(value))) == int(want), value
    rng = np.random.default_rng(1)
    values = (rng.standard_normal(20000) * np.exp(rng.uniform(-20, 12, 20000))).astype(np.float32)
    with np.errstate(over="ignore"):
        want = values.astype(np.float16).view(np.uint16)
    got = np.array([lib.oracle_float_to_half(float(v)) for v in values], np.uint16)
    np.testing.assert_array_equal(got, want)


def test_score_scale_is_correctly_rounded():
    assert np.float32(oracle.score_scale(128)).view(np.uint32) == 0x3DB504F3
