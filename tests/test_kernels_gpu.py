"""CUDA kernels vs the CPU oracle (bit-exact) and vs the reference's golden outputs.

Parity bars:
* sign/magnitude planes, fp16 key representatives, query planes and fp32
  query representatives, fp16/fp32 scores and top-k indices: bit-exact against
  the oracle (same IEEE arithmetic, same reduction orders, same tie-break);
* against the reference's own outputs: the reference tests' tolerances
  (planes exact, key reps 2e-3, query reps 2e-5, scores atol 0.15 / rtol 0.025);
* attention: fp32 kernel vs float64 oracle, max-abs 2e-2 and mean-abs 2e-3
  (the stated bf16 tolerance); in practice the error is ~1e-6.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from popkv_b200 import popkv as P
from popkv_b200 import popkv_cuda as C
from popkv_b200 import sparse_kernels as S
from tests.helpers import bits, from_bits, planes_to_numpy, random_keys, to_oracle

pytestmark = pytest.mark.gpu

GROUPS = (16, 32, 64)
DIMS = (32, 64, 96, 127, 128)
DTYPES = (torch.bfloat16, torch.float16, torch.float32)


def _oracle_pack(keys: torch.Tensor, tg: int, g: int, capacity=None):
    arr, tag = to_oracle(keys)
    return oracle.pack(arr, tag, token_group_size=tg, dim_group_size=g, token_capacity=capacity)


def _assert_planes_equal(packed, want, tokens):
    got = planes_to_numpy(packed)
    for name, a, b in zip(("sign", "mag", "low", "delta"), got, want):
        np.testing.assert_array_equal(a[:, :tokens], b[:, :tokens], err_msg=name)


@pytest.mark.parametrize("g", GROUPS)
@pytest.mark.parametrize("dim", DIMS)
@pytest.mark.parametrize("dtype", DTYPES)
def test_pack_matches_oracle(cuda_device, g, dim, dtype):
    gen = torch.Generator().manual_seed(1000 + g + dim)
    keys = random_keys(gen, (2, 37, dim), dtype, cuda_device)
    packed = C.pack_keys(keys, dim_group_size=g, token_capacity=40)
    _assert_planes_equal(packed, _oracle_pack(keys, 32, g), 37)


@pytest.mark.parametrize("g,tg", [(32, t) for t in (1, 5, 8, 10, 16, 32, 64, 125, 128, 500, 4096)]
                         + [(16, t) for t in (8, 16, 32, 64, 128)]
                         + [(64, t) for t in (8, 16, 32, 64, 128)])
def test_pack_token_groups_match_oracle(cuda_device, g, tg):
    gen = torch.Generator().manual_seed(tg * 7 + g)
    tokens = tg + 3 if tg < 1000 else 4100
    keys = random_keys(gen, (2, tokens, 128), torch.bfloat16, cuda_device)
    packed = C.pack_keys(keys, token_group_size=tg, dim_group_size=g)
    _assert_planes_equal(packed, _oracle_pack(keys, tg, g), tokens)


@pytest.mark.parametrize("g", GROUPS)
@pytest.mark.parametrize("dim", DIMS)
def test_pack_matches_reference_golden(cuda_device, golden, g, dim):
    tag = f"g{g}_d{dim}"
    keys = from_bits(golden[f"kenc/{tag}/k"], torch.bfloat16, cuda_device)
    packed = C.pack_keys(keys, dim_group_size=g)
    np.testing.assert_array_equal(packed[0].cpu().numpy(), golden[f"kenc/{tag}/sign"])
    np.testing.assert_array_equal(packed[1].cpu().numpy(), golden[f"kenc/{tag}/mag"])
    np.testing.assert_allclose(packed[2].float().cpu().numpy(), golden[f"kenc/{tag}/low"], atol=2e-3, rtol=2e-3)
    np.testing.assert_allclose(packed[3].float().cpu().numpy(), golden[f"kenc/{tag}/delta"], atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize("g,tg", [(16, 128), (64, 64), (32, 32), (16, 8), (32, 5)])
def test_incremental_append_matches_oracle(cuda_device, g, tg):
    """build_popkv_cache + append_popkv across every group boundary (reference test :355-372)."""
    gen = torch.Generator().manual_seed(41 + tg)
    keys = random_keys(gen, (2, tg - 1, 128), torch.bfloat16, cuda_device)
    cache = P.build_popkv_cache(keys, group_size=tg, dim_group_size=g, reserve_tokens=tg + 3)
    for _ in range(tg + 2):
        current = random_keys(gen, (2, 1, 128), torch.bfloat16, cuda_device)
        P.append_popkv(cache, current)
        keys = torch.cat((keys, current), dim=1)
        tokens = keys.shape[1]
        _assert_planes_equal(cache.packed, _oracle_pack(keys, tg, g), tokens)
        assert cache.token_count == tokens
        assert cache.sealed_tokens == (tokens // tg) * tg


@pytest.mark.parametrize("g", GROUPS)
@pytest.mark.parametrize("dim", DIMS)
@pytest.mark.parametrize("dtype", DTYPES)
def test_query_encode_matches_oracle(cuda_device, g, dim, dtype):
    gen = torch.Generator().manual_seed(17 + dim)
    q = torch.randn(2, 8, dim, generator=gen).to(dtype).to(cuda_device)
    got = C.query_encode(q, dim_group_size=g)
    arr, tag = to_oracle(q)
    want = oracle.query_encode(arr, tag, dim_group_size=g)
    for a, b in zip(got, want):
        np.testing.assert_array_equal(a.cpu().numpy(), b)


@pytest.mark.parametrize("g", GROUPS)
@pytest.mark.parametrize("dim", DIMS)
def test_query_encode_matches_reference_golden(cuda_device, golden, g, dim):
    tag = f"g{g}_d{dim}"
    q = from_bits(golden[f"qenc/{tag}/q"], torch.bfloat16, cuda_device)
    got = C.query_encode(q, dim_group_size=g)
    np.testing.assert_array_equal(got[0].cpu().numpy(), golden[f"qenc/{tag}/sign"])
    np.testing.assert_array_equal(got[1].cpu().numpy(), golden[f"qenc/{tag}/mag"])
    np.testing.assert_allclose(got[2].cpu().numpy(), golden[f"qenc/{tag}/low"], atol=2e-5, rtol=2e-5)
    np.testing.assert_allclose(got[3].cpu().numpy(), golden[f"qenc/{tag}/delta"], atol=2e-5, rtol=2e-5)


def test_query_encode_hand_case_and_empty_buckets(cuda_device, golden):
    q = torch.tensor([[[1.0, -1.0, 3.0, -3.0, 0.0]]], device=cuda_device)
    sign, mag, low, delta = C.query_encode(q, dim_group_size=32)
    assert int(sign.item()) == 0b10101 and int(mag.item()) == 0b01100
    assert float(low.item()) == float(np.float32(2.0) / np.float32(3.0))
    for tag in ("pos", "neg"):
        q = torch.from_numpy(golden[f"empty_{tag}/q"]).to(cuda_device)
        out = C.query_encode(q, dim_group_size=32)
        assert int(out[1].item()) == -1
        np.testing.assert_array_equal(out[2].cpu().numpy(), golden[f"empty_{tag}/low"])
        np.testing.assert_array_equal(out[3].cpu().numpy(), golden[f"empty_{tag}/delta"])


def _score_case(cuda_device, g, batch, tokens, q_heads=8, kv_heads=2, dim=128, seed=0,
                qdtype=torch.bfloat16, capacity=None):
    gen = torch.Generator().manual_seed(seed)
    keys = random_keys(gen, (kv_heads, tokens, dim), torch.bfloat16, cuda_device)
    q = torch.randn(batch, q_heads, dim, generator=gen).to(qdtype).to(cuda_device)
    mapping = torch.arange(q_heads, device=cuda_device) // (q_heads // kv_heads)
    packed = C.pack_keys(keys, dim_group_size=g, token_capacity=capacity or tokens + 5)
    return keys, q, mapping, packed


@pytest.mark.parametrize("g", GROUPS)
@pytest.mark.parametrize("batch,tokens", [(1, 37), (2, 257), (1, 1), (3, 1500)])
def test_score_encoded_matches_oracle_bit_exact(cuda_device, g, batch, tokens):
    keys, q, mapping, packed = _score_case(cuda_device, g, batch, tokens, seed=tokens + g)
    enc = C.query_encode(q, dim_group_size=g)
    got = C.score_encoded(enc, packed, head_to_kv=mapping, tokens=tokens, dim_group_size=g)
    assert got.dtype == torch.float16 and tuple(got.shape) == (batch, 8, tokens)
    penc = tuple(t.cpu().numpy() for t in enc)
    ppk = planes_to_numpy(packed)
    _, want16 = oracle.score(penc, ppk, head_to_kv=mapping.cpu().numpy(), tokens=tokens,
                             dim_group_size=g, head_dim=128)
    np.testing.assert_array_equal(bits(got), want16)
    raw = C.score(q, packed, head_to_kv=mapping, tokens=tokens, dim_group_size=g)
    np.testing.assert_array_equal(bits(raw), want16)


@pytest.mark.parametrize("g", GROUPS)
@pytest.mark.parametrize("group_heads", (1, 2, 4, 8, 16))
def test_score_gqa_group_sizes(cuda_device, g, group_heads):
    kv_heads = 2
    keys, q, mapping, packed = _score_case(cuda_device, g, 1, 300, q_heads=kv_heads * group_heads,
                                           kv_heads=kv_heads, seed=group_heads)
    got = C.score(q, packed, head_to_kv=mapping, tokens=300, dim_group_size=g)
    arr, tag = to_oracle(q)
    penc = oracle.query_encode(arr, tag, dim_group_size=g)
    _, want16 = oracle.score(penc, planes_to_numpy(packed), head_to_kv=mapping.cpu().numpy(),
                             tokens=300, dim_group_size=g, head_dim=128)
    np.testing.assert_array_equal(bits(got), want16)


@pytest.mark.parametrize("g", GROUPS)
@pytest.mark.parametrize("dim", (32, 64, 96, 127))
def test_generic_head_dim_scores_fp32_bit_exact(cuda_device, g, dim):
    keys, q, mapping, packed = _score_case(cuda_device, g, 1, 37, dim=dim, seed=dim)
    got = C.score(q, packed, head_to_kv=mapping, tokens=37, dim_group_size=g)
    assert got.dtype == torch.float32
    arr, tag = to_oracle(q)
    penc = oracle.query_encode(arr, tag, dim_group_size=g)
    want32, _ = oracle.score(penc, planes_to_numpy(packed), head_to_kv=mapping.cpu().numpy(),
                             tokens=37, dim_group_size=g, head_dim=dim)
    np.testing.assert_array_equal(got.cpu().numpy().view(np.uint32), want32.view(np.uint32))


@pytest.mark.parametrize("g", GROUPS)
@pytest.mark.parametrize("dim", DIMS)
def test_scores_match_reference_golden(cuda_device, golden, g, dim):
    tag = f"g{g}_d{dim}"
    keys = from_bits(golden[f"kenc/{tag}/k"], torch.bfloat16, cuda_device)
    q = from_bits(golden[f"qenc/{tag}/q"], torch.bfloat16, cuda_device)
    mapping = torch.from_numpy(golden["mapping8"]).to(cuda_device)
    packed = C.pack_keys(keys, dim_group_size=g)
    got = C.score(q, packed, head_to_kv=mapping, tokens=37, dim_group_size=g)
    assert got.dtype == (torch.float16 if dim == 128 else torch.float32)
    np.testing.assert_allclose(got.float().cpu().numpy(), golden[f"score/{tag}"], atol=0.15, rtol=0.025)


@pytest.mark.parametrize("g", GROUPS)
@pytest.mark.parametrize("batch,tokens,group_heads,qdtype", [
    (1, 1, 4, torch.bfloat16), (1, 127, 4, torch.bfloat16), (2, 129, 2, torch.float16),
    (1, 4097, 1, torch.float32), (3, 1000, 4, torch.bfloat16), (1, 32768, 4, torch.bfloat16)])
def test_tensor_core_score_matches_popcount_kernel(cuda_device, g, batch, tokens, group_heads, qdtype):
    """popkv_score_tc (tcgen05 int8 counts) == popkv_score_encoded (popcounts), bit for bit."""
    keys, q, mapping, packed = _score_case(cuda_device, g, batch, tokens, q_heads=2 * group_heads,
                                           kv_heads=2, seed=tokens + 7 * g, qdtype=qdtype)
    mma = C.score(q, packed, head_to_kv=mapping, tokens=tokens, dim_group_size=g, kernel="tensor_core")
    enc = C.query_encode(q, dim_group_size=g)
    popc = C.score_encoded(enc, packed, head_to_kv=mapping, tokens=tokens, dim_group_size=g)
    assert torch.equal(mma.view(torch.int16), popc.view(torch.int16))
    import ctypes
    from popkv_b200 import _lib
    timeouts = ctypes.c_uint32(0)
    _lib.check(_lib.lib().popkv_score_tc_timeouts(ctypes.byref(timeouts)))
    assert timeouts.value == 0
    if tokens <= 1000:
        arr, tag = to_oracle(q)
        penc = oracle.query_encode(arr, tag, dim_group_size=g)
        _, want = oracle.score(penc, planes_to_numpy(packed), head_to_kv=mapping.cpu().numpy(),
                               tokens=tokens, dim_group_size=g, head_dim=128)
        np.testing.assert_array_equal(bits(mma), want)


@pytest.fixture
def fp8_scorer():
    """The fp8 tensor-core scorer for every shape it applies to (the automatic
    choice takes the popcount scorer for small shapes), restored afterwards."""
    C.set_score_dispatch("fp8")
    yield
    C.set_score_dispatch("auto")


@pytest.mark.parametrize("g", GROUPS)
@pytest.mark.parametrize("batch,tokens,group_heads,qdtype,capacity", [
    (1, 1, 4, torch.bfloat16, 128), (1, 127, 4, torch.bfloat16, 132), (1, 129, 4, torch.float16, 256),
    (2, 300, 2, torch.float32, 304), (1, 777, 1, torch.bfloat16, 780), (3, 1000, 4, torch.bfloat16, 1024),
    (1, 515, 5, torch.bfloat16, 520), (2, 260, 8, torch.float16, 264), (1, 1500, 3, torch.bfloat16, 1504),
    (1, 32768, 4, torch.bfloat16, 32768)])
def test_fp8_score_matches_popcount_kernel_and_oracle(fp8_scorer, cuda_device, g, batch, tokens, group_heads,
                                                      qdtype, capacity):
    """popkv_score (fp8 tensor-core counts, every capacity here 16-byte aligned per row)
    == popkv_score_popcount == popkv_score_encoded, bit for bit, and == the oracle."""
    kv_heads = 2
    keys, q, mapping, packed = _score_case(cuda_device, g, batch, tokens, q_heads=kv_heads * group_heads,
                                           kv_heads=kv_heads, seed=tokens + 11 * g + group_heads,
                                           qdtype=qdtype, capacity=capacity)
    f8 = C.score(q, packed, head_to_kv=mapping, tokens=tokens, dim_group_size=g)
    popc = C.score(q, packed, head_to_kv=mapping, tokens=tokens, dim_group_size=g, kernel="popcount")
    enc = C.query_encode(q, dim_group_size=g)
    f8_enc = C.score_encoded(enc, packed, head_to_kv=mapping, tokens=tokens, dim_group_size=g)
    assert torch.equal(f8.view(torch.int16), popc.view(torch.int16))
    assert torch.equal(f8_enc.view(torch.int16), popc.view(torch.int16))
    import ctypes
    from popkv_b200 import _lib
    timeouts = ctypes.c_uint32(0)
    _lib.check(_lib.lib().popkv_score_tc_timeouts(ctypes.byref(timeouts)))
    assert timeouts.value == 0
    if tokens <= 1500:
        arr, tag = to_oracle(q)
        penc = oracle.query_encode(arr, tag, dim_group_size=g)
        _, want = oracle.score(penc, planes_to_numpy(packed), head_to_kv=mapping.cpu().numpy(),
                               tokens=tokens, dim_group_size=g, head_dim=128)
        np.testing.assert_array_equal(bits(f8), want)


def test_fp8_score_special_planes(fp8_scorer, cuda_device):
    """All-sign, no-sign, all-magnitude and empty-bucket planes (counts at +-16/32/64)."""
    for g in GROUPS:
        keys = torch.zeros(2, 256, 128, dtype=torch.bfloat16, device=cuda_device)
        keys[0, 0::4] = 1.0
        keys[0, 1::4] = -1.0
        keys[1, 2::4] = torch.linspace(-3, 3, 128, device=cuda_device).to(torch.bfloat16)
        keys[1, 3::4, ::2] = 4.0
        q = torch.zeros(1, 8, 128, dtype=torch.bfloat16, device=cuda_device)
        q[0, 0] = 1.0
        q[0, 1] = -1.0
        q[0, 2, ::3] = 2.0
        q[0, 3] = torch.linspace(-1, 1, 128, device=cuda_device).to(torch.bfloat16)
        q[0, 4:] = torch.randn(4, 128, generator=torch.Generator().manual_seed(g)).to(torch.bfloat16).to(cuda_device)
        mapping = torch.arange(8, device=cuda_device) // 4
        packed = C.pack_keys(keys, dim_group_size=g, token_capacity=256)
        f8 = C.score(q, packed, head_to_kv=mapping, tokens=256, dim_group_size=g)
        popc = C.score(q, packed, head_to_kv=mapping, tokens=256, dim_group_size=g, kernel="popcount")
        assert torch.equal(f8.view(torch.int16), popc.view(torch.int16)), g


def test_tensor_core_score_rejects_unsupported(cuda_device):
    keys, q, mapping, packed = _score_case(cuda_device, 16, 1, 64, q_heads=16, kv_heads=2, seed=1)
    with pytest.raises(RuntimeError, match="at most 4 query heads"):
        C.score(q, packed, head_to_kv=mapping, tokens=64, dim_group_size=16, kernel="tensor_core")
    with pytest.raises(ValueError, match="kernel must be"):
        C.score(q, packed, head_to_kv=mapping, tokens=64, dim_group_size=16, kernel="mma")


def test_score_dim_kernel_variants_agree(cuda_device):
    """g64-u32 and g64-u64 name the same arithmetic (reference test :320-331)."""
    keys, q, mapping, packed = _score_case(cuda_device, 64, 1, 257, seed=33)
    u32 = C.score(q, packed, head_to_kv=mapping, tokens=257, dim_group_size=64, dim_kernel="g64-u32")
    u64 = C.score(q, packed, head_to_kv=mapping, tokens=257, dim_group_size=64, dim_kernel="g64-u64")
    assert torch.equal(u32, u64)


def _tie_heavy_scores(gen, rows, tokens, levels=None):
    x = torch.randn(rows, tokens, generator=gen)
    if levels:
        x = torch.round(x * levels) / levels
    return x


@pytest.mark.parametrize("tokens", (1, 2, 100, 1000, 4096, 32768, 33024, 49152, 65536, 98304, 131072))
@pytest.mark.parametrize("dtype", (torch.float16, torch.float32))
def test_topk_matches_oracle(cuda_device, tokens, dtype):
    gen = torch.Generator().manual_seed(tokens)
    rows = 4 if tokens > 40000 else 8
    scores = _tie_heavy_scores(gen, rows, tokens, levels=8 if tokens % 2 == 0 else None)
    scores = scores.to(dtype).to(cuda_device)
    host = bits(scores) if dtype == torch.float16 else scores.cpu().numpy()
    for k in sorted({0, 1, min(tokens, 511), tokens // 2, max(tokens - 1, 0), tokens}):
        got = C.topk(scores, k, current_index=tokens)
        want = oracle.topk(host, k)
        np.testing.assert_array_equal(got[:, :k].cpu().numpy(), want)
        assert torch.all(got[:, k] == tokens)


@pytest.mark.parametrize("rows,tokens", [(1, 131072), (3, 65536), (32, 32768), (32, 33024), (64, 8191),
                                         (200, 777), (160, 70000), (32, 40000), (48, 49152)])
def test_topk_all_equal_and_row_counts(cuda_device, rows, tokens):
    """Every key equal (all winners are ties, taken in index order) and many cluster shapes."""
    gen = torch.Generator().manual_seed(rows)
    flat = torch.full((rows, tokens), 0.5, dtype=torch.float16, device=cuda_device)
    mixed = _tie_heavy_scores(gen, rows, tokens, levels=2).half().to(cuda_device)
    for scores in (flat, mixed):
        for k in sorted({1, tokens // 3, tokens - 1, tokens}):
            got = C.topk(scores, k, current_index=tokens)
            want = oracle.topk(bits(scores), k)
            np.testing.assert_array_equal(got[:, :k].cpu().numpy(), want)
            assert torch.all(got[:, k] == tokens)


@pytest.mark.parametrize("rows,tokens", [(32, 32771), (32, 45000), (40, 49152)])
def test_topk_rows_just_past_32k_keys(cuda_device, rows, tokens):
    """The decoder's sparse layers (32 rows of a few tokens over 32768, 4 CTAs at
    24 keys per thread): the budget's k and a tie-free and a tie-heavy row set."""
    gen = torch.Generator().manual_seed(tokens)
    for levels in (None, 4):
        scores = _tie_heavy_scores(gen, rows, tokens, levels=levels).half().to(cuda_device)
        for k in (4095, tokens - 1):
            got = C.topk(scores, k, current_index=tokens)
            want = oracle.topk(bits(scores), k)
            np.testing.assert_array_equal(got[:, :k].cpu().numpy(), want)
            assert torch.all(got[:, k] == tokens)


def test_topk_special_values(cuda_device):
    vals = [0.0, -0.0, 1.0, -1.0, float("inf"), float("-inf"), float("nan"), 65504.0, -65504.0,
            6e-8, -6e-8, 0.0, -0.0, 1.0]
    scores = torch.tensor([vals * 3], dtype=torch.float16, device=cuda_device)
    for k in range(scores.shape[1] + 1):
        got = C.topk(scores, k)
        want = oracle.topk(bits(scores), k)
        np.testing.assert_array_equal(got.cpu().numpy(), want)


def test_topk_strided_rows_and_batch_axes(cuda_device):
    gen = torch.Generator().manual_seed(5)
    full = torch.randn(2, 4, 300, generator=gen).half().to(cuda_device)
    view = full[..., :257]
    got = P.select_tokens(view, budget=64, prefix_tokens=257)
    assert tuple(got.shape) == (2, 4, 64)
    want = oracle.select_with_current(bits(view.contiguous()), 64, 257)
    np.testing.assert_array_equal(got.cpu().numpy(), want)


def test_topk_matches_torch_topk_modulo_ties(cuda_device, golden):
    scores = from_bits(golden["topk/scores16"], torch.float16, cuda_device)
    values = scores.float().cpu().numpy()
    for k in (1, 255, 511, 1024):
        mine = C.topk(scores, k).cpu().numpy()
        want = golden[f"topk/k{k}"].astype(np.int64)
        for row in range(scores.shape[1]):
            v = values[0, row]
            kth = np.sort(v[want[0, row]])[0]
            assert set(mine[0, row][v[mine[0, row]] > kth]) == set(want[0, row][v[want[0, row]] > kth])
            assert (v[mine[0, row]] == kth).sum() == (v[want[0, row]] == kth).sum()


def _attn_inputs(cuda_device, *, q_heads=8, kv_heads=2, tokens=700, dim=128, selected=300,
                 dtype=torch.bfloat16, batch=None, seed=0, valid=False, pad=11):
    gen = torch.Generator().manual_seed(seed)
    lead = () if batch is None else (batch,)
    queries = torch.randn(*lead, q_heads, dim, generator=gen).to(dtype).to(cuda_device)
    kstore = torch.randn(*lead, kv_heads, tokens + pad, dim, generator=gen).to(dtype).to(cuda_device)
    vstore = torch.randn(*lead, kv_heads, tokens + pad, dim, generator=gen).to(dtype).to(cuda_device)
    keys, values = kstore[..., :tokens, :], vstore[..., :tokens, :]
    cur_k = torch.randn(*lead, kv_heads, dim, generator=gen).to(dtype).to(cuda_device)
    cur_v = torch.randn(*lead, kv_heads, dim, generator=gen).to(dtype).to(cuda_device)
    mapping = torch.arange(q_heads, device=cuda_device) // (q_heads // kv_heads)
    indices = torch.randint(tokens, (*lead, q_heads, selected), generator=gen).to(cuda_device)
    indices[..., -1] = tokens
    mask = None
    if valid:
        mask = torch.ones_like(indices, dtype=torch.bool)
        mask[..., -7:-1] = False
        mask[..., 256:272] = False  # a fully masked 16-slot tile at a split start
    return queries, keys, values, cur_k, cur_v, indices, mapping, mask


def _oracle_attention(queries, keys, values, cur_k, cur_v, indices, mapping, mask, split):
    q, qt = to_oracle(queries)
    k, kt = to_oracle(keys)
    v, _ = to_oracle(values)
    ck, _ = to_oracle(cur_k)
    cv, _ = to_oracle(cur_v)
    return oracle.attn_partial(q, qt, k, v, kt, ck, cv, indices.cpu().numpy(), mapping.cpu().numpy(),
                               None if mask is None else mask.cpu().numpy(), split_tokens=split)


_OUT_EPS = {torch.float32: 0.0, torch.float16: 2.0 ** -11, torch.bfloat16: 2.0 ** -8}


def _check_attention(out, want, dtype=torch.float32):
    err = np.abs(out.astype(np.float64) - want)
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, (err.max(), err.mean())
    # fp32 arithmetic: beyond the output's own rounding, the error stays near 1e-5.
    assert np.all(err <= 2e-5 + np.abs(want) * _OUT_EPS[dtype]), err.max()


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("valid", (False, True))
@pytest.mark.parametrize("split", (256, 64, 512))
def test_split_attention_matches_oracle(cuda_device, dtype, valid, split):
    args = _attn_inputs(cuda_device, dtype=dtype, valid=valid, seed=split)
    partials = S.indexed_attention_split_partial(*args[:6], args[6], args[7], split_tokens=split)
    want = _oracle_attention(*args, split)
    got = partials.cpu().numpy()
    assert got.shape == want.shape
    live = np.isfinite(want[..., 0])
    np.testing.assert_array_equal(np.isfinite(got[..., 0]), live)
    np.testing.assert_allclose(got[..., 0][live], want[..., 0][live], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(got[..., 1:], want[..., 1:], atol=1e-3, rtol=1e-4)
    merged = S.indexed_attention_split_merge(partials, args[0])
    assert merged.dtype == dtype
    _check_attention(merged.float().cpu().numpy(), oracle.attn_merge(want), dtype)


@pytest.mark.parametrize("dim", (64, 96))
def test_split_attention_generic_head_dim(cuda_device, dim):
    args = _attn_inputs(cuda_device, dim=dim, valid=True, seed=dim)
    out = S.indexed_attention_split(*args[:6], args[6], args[7], split_tokens=256)
    want = oracle.attn_merge(_oracle_attention(*args, 256))
    _check_attention(out.float().cpu().numpy(), want, torch.bfloat16)


def test_split_attention_matches_reference_golden(cuda_device, golden):
    dev = cuda_device
    prefix = int(golden["attn/prefix_tokens"])
    kstore = from_bits(golden["attn/k_store"], torch.bfloat16, dev)
    vstore = from_bits(golden["attn/v_store"], torch.bfloat16, dev)
    args = (from_bits(golden["attn/q"], torch.bfloat16, dev), kstore[:, :prefix], vstore[:, :prefix],
            from_bits(golden["attn/cur_k"], torch.bfloat16, dev),
            from_bits(golden["attn/cur_v"], torch.bfloat16, dev),
            torch.from_numpy(golden["attn/indices"]).to(dev),
            torch.from_numpy(golden["attn/mapping"]).to(dev),
            torch.from_numpy(golden["attn/valid"]).to(dev))
    partials = S.indexed_attention_split_partial(*args, split_tokens=256)
    np.testing.assert_allclose(partials.cpu().numpy(), golden["attn/partials"], atol=1e-4, rtol=1e-4)
    out = S.indexed_attention_split_merge(partials, torch.empty(8, 128, device=dev))
    np.testing.assert_allclose(out.cpu().numpy(), golden["attn/merged"], atol=1e-5, rtol=1e-4)
    np.testing.assert_allclose(out.cpu().numpy(), golden["attn/dense"], atol=1e-5, rtol=1e-4)


def test_batched_attention_matches_oracle(cuda_device):
    args = _attn_inputs(cuda_device, batch=3, valid=True, seed=9)
    partials = S.indexed_attention_split_partial_batched(*args[:6], args[6], args[7])
    out = S.indexed_attention_split_merge_batched(partials, torch.float32).cpu().numpy()
    for b in range(3):
        one = [a[b] if a is not None and a is not args[6] else a for a in args]
        want = oracle.attn_merge(_oracle_attention(*one, 256))
        _check_attention(out[b], want)


def test_attention_rejects_bad_arguments(cuda_device):
    args = _attn_inputs(cuda_device)
    with pytest.raises(ValueError, match="multiple of 16"):
        S.indexed_attention_split_partial(*args[:6], args[6], split_tokens=100)
    with pytest.raises(ValueError, match="indices must be"):
        S.indexed_attention_split_partial(*args[:5], args[5][:4], args[6])
    with pytest.raises(ValueError, match="valid mask"):
        S.indexed_attention_split_partial(*args[:6], args[6], torch.ones(3, 3, dtype=torch.bool,
                                                                            device=cuda_device))


@pytest.mark.parametrize("valid", (False, True))
def test_partial_merge_single_launch_matches_two_launches(cuda_device, valid):
    """popkv_attn_partial_merge (last CTA merges) == popkv_attn_partial + popkv_attn_merge."""
    from popkv_b200 import _lib
    args = _attn_inputs(cuda_device, valid=valid, seed=77, selected=1000)
    q, keys, values, ck, cv, idx, mapping, mask = args
    partials = S.indexed_attention_split_partial(*args[:6], mapping, mask)
    want = S.indexed_attention_split_merge(partials, q)
    out = torch.empty_like(q)
    scratch = torch.empty_like(partials)
    counters = torch.zeros(q.shape[0], dtype=torch.int32, device=cuda_device)
    idx = idx.contiguous()
    m = None if mask is None else mask.to(torch.uint8).contiguous()
    for _ in range(2):  # the counters reset themselves
        _lib.check(_lib.lib().popkv_attn_partial_merge(
            _lib.ptr(q), _lib.BF16, 1, q.shape[0], 128, _lib.ptr(keys), _lib.ptr(values), _lib.BF16,
            keys.shape[0], keys.shape[1], 0, keys.stride(0), keys.stride(1), 0, values.stride(0),
            values.stride(1), _lib.ptr(ck), _lib.ptr(cv), _lib.ptr(idx), idx.shape[1], _lib.ptr(m),
            _lib.ptr(mapping), 256, _lib.ptr(scratch), _lib.ptr(counters), _lib.ptr(out), _lib.BF16,
            _lib.stream_of(cuda_device)))
        torch.cuda.synchronize()
        assert int(counters.abs().sum()) == 0
        torch.testing.assert_close(out.float(), want.float(), atol=1e-2, rtol=0)
        assert (out.float() - want.float()).abs().max().item() <= 2 ** -7


@pytest.mark.parametrize("g", GROUPS)
@pytest.mark.parametrize("tokens,budget", [(32768, 4096), (3000, 256), (100, 1000), (65536, 4096),
                                           (777, 500), (131072, 4096), (5000, 1)])
def test_score_hist_and_topk_hist_match_separate_kernels(cuda_device, g, tokens, budget):
    """popkv_score_hist + popkv_topk_hist == popkv_score + popkv_topk, and the histogram is re-zeroed."""
    from popkv_b200 import _lib
    keys, q, mapping, packed = _score_case(cuda_device, g, 1, tokens, q_heads=32, kv_heads=8,
                                           seed=tokens + g)
    want_scores = C.score(q, packed, head_to_kv=mapping, tokens=tokens, dim_group_size=g)
    k = min(budget - 1, tokens)
    want_idx = C.topk(want_scores, k, current_index=tokens)
    scores = torch.empty_like(want_scores)
    hist = torch.zeros(32, 2048, dtype=torch.int32, device=cuda_device)
    idx = torch.empty(1, 32, k + 1, dtype=torch.int64, device=cuda_device)
    cap = packed[0].shape[1]
    for _ in range(2):
        _lib.check(_lib.lib().popkv_score_hist(
            _lib.ptr(q), _lib.BF16, 1, 32, *(_lib.ptr(t) for t in packed), 8, cap, _lib.ptr(mapping),
            tokens, g, _lib.ptr(scores), _lib.ptr(hist), _lib.stream_of(cuda_device)))
        torch.cuda.synchronize()
        assert int(hist.sum()) == 32 * tokens
        _lib.check(_lib.lib().popkv_topk_hist(
            _lib.ptr(scores), _lib.ptr(hist), 32, tokens, tokens, k, tokens, _lib.ptr(idx), k + 1,
            _lib.stream_of(cuda_device)))
        torch.cuda.synchronize()
        assert torch.equal(scores, want_scores)
        assert torch.equal(idx, want_idx)
        assert int(hist.abs().sum()) == 0


def test_experimental_topk_hook_shape_and_selection(cuda_device):
    """popkv.topk as LlamaSparseDecoder.experimental_topk (popkv.py:1091-1093): fp16 [B, QH, T]
    -> int64 [B, QH, k], the same tokens as select_tokens without its current slot."""
    gen = torch.Generator().manual_seed(5)
    scores = torch.randn(1, 32, 5000, generator=gen).to(torch.float16).to(cuda_device)
    k = 511
    got = P.topk(scores, k)
    assert got.dtype == torch.int64 and tuple(got.shape) == (1, 32, k)
    with_current = P.select_tokens(scores, budget=k + 1, prefix_tokens=5000)
    assert torch.equal(got[0], with_current[0, :, :k])
    # The reference then indexes [0] and appends the current slot itself.
    assert torch.equal(P._append_current(got[0], 5001), with_current[0])  # num_tokens = prefix + 1
