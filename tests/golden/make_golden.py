"""Generate tests/golden/popkv_golden.npz from the reference implementation.

Run in a container where the reference checkout is available (read-only is
fine): ``python tests/golden/make_golden.py --reference /path/to/PopKV``.
It imports the reference's own readable oracles (popkv.py:462-735,
popkv.py:287) and launches its Triton split-attention kernels under
``TRITON_INTERPRET=1`` (sparse_kernels.py:237-318), and stores their inputs and
outputs.  The fixture is what pins the CPU oracle in ``oracle/`` to the
reference; the tests only read the .npz, never the reference itself.

Cases mirror the reference tests: tests/test_popkv.py:184-197 (hand-computed
query, empty buckets), :200-211 and :213-234 (every dim group and head-dim
tail), :236-246 and :334-352 (token groups), :262-273 (popcount
decomposition), :276-300 (key planes and scores), :355-372 (incremental
append across group boundaries), :47-50 (current-slot reservation), and
tests/test_sparse_kernels.py:118-141 (split attention vs dense attention over
the same indices, with masked slots).
"""
from __future__ import annotations

import argparse
import math
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def bf16_bits(t):
    import torch
    return t.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def f16_bits(t):
    import torch
    return t.to(torch.float16).contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("POPKV_REFERENCE"),
                        required="POPKV_REFERENCE" not in os.environ,
                        help="checkout of the reference (kw78999/PopKV) to import; or set POPKV_REFERENCE")
    parser.add_argument("--out", default=str(HERE / "popkv_golden.npz"))
    args = parser.parse_args()
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, args.reference)
    import torch
    import popkv  # the reference module
    import sparse_kernels  # the reference module (Triton kernels, interpreted on CPU)

    torch.manual_seed(0)
    gold: dict[str, np.ndarray] = {}

    # Hand-computable query (tests/test_popkv.py:184-190) and empty buckets (:192-197).
    q = torch.tensor([[[1.0, -1.0, 3.0, -3.0, 0.0]]])
    for name, value in zip(("sign", "mag", "low", "delta"), popkv.reference_query_encode(q, 32)):
        gold[f"hand/{name}"] = value.numpy()
    gold["hand/q"] = q.numpy()
    for tag, value in (("pos", 2.0), ("neg", -2.0)):
        q = torch.full((1, 1, 32), value)
        for name, out in zip(("sign", "mag", "low", "delta"), popkv.reference_query_encode(q, 32)):
            gold[f"empty_{tag}/{name}"] = out.numpy()
        gold[f"empty_{tag}/q"] = q.numpy()

    mapping = torch.arange(8) // 4
    gold["mapping8"] = mapping.numpy()
    gen = torch.Generator().manual_seed(17)
    for group in (16, 32, 64):
        for dim in (32, 64, 96, 127, 128):
            tag = f"g{group}_d{dim}"
            query = torch.randn(1, 8, dim, generator=gen).to(torch.bfloat16)
            keys = torch.randn(2, 37, dim, generator=gen).to(torch.bfloat16)
            gold[f"qenc/{tag}/q"] = bf16_bits(query)
            for name, out in zip(("sign", "mag", "low", "delta"),
                                 popkv.reference_query_encode(query, group)):
                gold[f"qenc/{tag}/{name}"] = out.numpy()
            gold[f"kenc/{tag}/k"] = bf16_bits(keys)
            for name, out in zip(("sign", "mag", "low", "delta"),
                                 popkv.reference_key_encode(keys, dim_group_size=group)):
                gold[f"kenc/{tag}/{name}"] = out.numpy()
            gold[f"score/{tag}"] = popkv.popkv_reference_scores(
                query, keys, head_to_kv=mapping, dim_group_size=group).numpy()

    # Token groups, including non-specialized sizes for G32 (tests/test_popkv.py:334-352)
    # and every specialized size for G16/G64.
    for group, sizes in ((32, (5, 8, 10, 16, 32, 64, 125, 128, 500)), (16, (8, 16, 32, 64, 128)),
                         (64, (8, 16, 32, 64, 128))):
        for tg in sizes:
            tag = f"g{group}_tg{tg}"
            keys = torch.randn(2, tg + 3, 128, generator=gen).to(torch.bfloat16)
            query = torch.randn(1, 8, 128, generator=gen).to(torch.bfloat16)
            gold[f"tg/{tag}/k"] = bf16_bits(keys)
            gold[f"tg/{tag}/q"] = bf16_bits(query)
            for name, out in zip(("sign", "mag", "low", "delta"),
                                 popkv.reference_key_encode(keys, dim_group_size=group,
                                                            token_group_size=tg)):
                gold[f"tg/{tag}/{name}"] = out.numpy()
            gold[f"tg/{tag}/score"] = popkv.popkv_reference_scores(
                query, keys, head_to_kv=mapping, group_size=tg, dim_group_size=group).numpy()

    # Popcount decomposition == direct reconstruction (tests/test_popkv.py:262-273).
    query = torch.tensor([[[3., -1., 0., -3., 1., -2., 2., 0.]]]).repeat(1, 1, 8)
    keys = torch.stack((query[0], -query[0]), dim=1)
    gold["bitwise/q"] = query.numpy()
    gold["bitwise/k"] = keys.numpy()
    for group in (16, 32, 64):
        gold[f"bitwise/g{group}"] = popkv.popkv_reference_bitwise_scores(
            query, keys, head_to_kv=torch.tensor([0]), dim_group_size=group).numpy()
        gold[f"bitwise/direct_g{group}"] = popkv.popkv_reference_scores(
            query, keys, head_to_kv=torch.tensor([0]), dim_group_size=group).numpy()

    # Current-slot reservation (tests/test_popkv.py:47-50).
    gold["append_current/in"] = np.array([[4, 7], [2, 9]], np.int64)
    gold["append_current/out"] = popkv._append_current(torch.tensor([[4, 7], [2, 9]]), 12).numpy()

    # torch.topk(sorted=False) on fp16 scores: the selection the reference decoder makes
    # (popkv.py:1094-1098).  Scores are the reference's reconstructed scores rounded to fp16.
    query = torch.randn(1, 8, 128, generator=gen)
    keys = torch.randn(2, 2048, 128, generator=gen)
    scores16 = popkv.popkv_reference_scores(query, keys, head_to_kv=mapping, group_size=64,
                                            dim_group_size=64).to(torch.float16)
    gold["topk/scores16"] = f16_bits(scores16)
    for k in (1, 255, 511, 1024):
        chosen = torch.topk(scores16, k=k, dim=-1, sorted=False).indices
        gold[f"topk/k{k}"] = np.sort(chosen.numpy(), axis=-1).astype(np.int16)

    # Split attention (sparse_kernels.py:321-401), interpreted on CPU, with masked slots,
    # a strided prefix view and the current slot (tests/test_sparse_kernels.py:118-141).
    q_heads, kv_heads, tokens, dim, selected = 8, 2, 320, 128, 300
    queries = torch.randn(q_heads, dim, generator=gen).to(torch.bfloat16)
    key_store = torch.randn(kv_heads, tokens + 13, dim, generator=gen).to(torch.bfloat16)
    value_store = torch.randn(kv_heads, tokens + 13, dim, generator=gen).to(torch.bfloat16)
    keys, values = key_store[:, :tokens], value_store[:, :tokens]
    cur_k = torch.randn(kv_heads, dim, generator=gen).to(torch.bfloat16)
    cur_v = torch.randn(kv_heads, dim, generator=gen).to(torch.bfloat16)
    amap = torch.arange(q_heads) // 4
    indices = torch.randint(tokens, (q_heads, selected), generator=gen)
    indices[:, -1] = tokens
    valid = torch.ones_like(indices, dtype=torch.bool)
    valid[:, -7:-1] = False
    splits = math.ceil(selected / 256)
    partials = torch.empty(q_heads, splits, dim + 2, dtype=torch.float32)
    sparse_kernels._indexed_attention_split_kernel[(q_heads, splits)](
        queries, keys, values, cur_k, cur_v, indices, valid.to(torch.int8), amap, partials,
        tokens, selected, splits,
        stride_kh=keys.stride(0), stride_kt=keys.stride(1),
        stride_vh=values.stride(0), stride_vt=values.stride(1),
        q_heads=q_heads, head_dim=dim, scale=1.0 / math.sqrt(dim), HAS_VALID=True,
        SPLIT_T=256, BLOCK_T=16, BLOCK_D=128, STATE_D=dim + 2)
    merged = torch.empty(q_heads, dim, dtype=torch.float32)
    sparse_kernels._indexed_attention_merge_kernel[(q_heads,)](
        partials, merged, splits, head_dim=dim, BLOCK_S=2, BLOCK_D=128, STATE_D=dim + 2)
    sys.path.insert(0, str(Path(args.reference) / "tests"))
    from test_sparse_kernels import materialized_attention  # reference test helper
    dense = materialized_attention(queries.float(), keys.float(), values.float(), cur_k.float(),
                                   cur_v.float(), indices, amap, valid)
    gold["attn/q"] = bf16_bits(queries)
    gold["attn/k_store"] = bf16_bits(key_store)
    gold["attn/v_store"] = bf16_bits(value_store)
    gold["attn/prefix_tokens"] = np.array(tokens, np.int64)
    gold["attn/cur_k"] = bf16_bits(cur_k)
    gold["attn/cur_v"] = bf16_bits(cur_v)
    gold["attn/indices"] = indices.numpy()
    gold["attn/valid"] = valid.numpy()
    gold["attn/mapping"] = amap.numpy()
    gold["attn/partials"] = partials.numpy()
    gold["attn/merged"] = merged.numpy()
    gold["attn/dense"] = dense.numpy()

    np.savez_compressed(args.out, **gold)
    size = Path(args.out).stat().st_size
    print(f"wrote {args.out}: {len(gold)} arrays, {size / 1024:.1f} KiB")


if __name__ == "__main__":
    main()
