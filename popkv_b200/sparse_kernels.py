"""Drop-in replacement of the reference's split sparse attention (sparse_kernels.py).

``indexed_attention_split_partial`` / ``_merge`` / ``indexed_attention_split``
keep the reference's signatures, validation messages and output layout
(sparse_kernels.py:321-401), and run the sm_100a kernels of
``libpopkv_b200.so``.  Batched forms (``*_batched``) take a leading batch axis,
which the reference's batch-1 kernels lack.

QUEST page scoring/selection belongs to a comparison method outside this
package and raises NotImplementedError.
"""
from __future__ import annotations

import math

import torch

from . import _lib


def _check_common(queries, prefix_keys, prefix_values, current_keys, current_values, indices,
                  head_to_kv, valid_mask, split_tokens, batched: bool):
    q_rank, kv_rank = (3, 4) if batched else (2, 3)
    if queries.ndim != q_rank or prefix_keys.ndim != kv_rank or prefix_values.shape != prefix_keys.shape:
        raise ValueError("invalid indexed-attention tensor ranks or K/V shapes")
    if indices.ndim != q_rank or tuple(indices.shape[:-1]) != tuple(queries.shape[:-1]):
        raise ValueError("indices must be [query heads, selected tokens]")
    if valid_mask is not None and valid_mask.shape != indices.shape:
        raise ValueError("valid mask must match indices")
    if split_tokens <= 0 or split_tokens % 16:
        raise ValueError("split_tokens must be a positive multiple of 16")
    if not queries.is_cuda or any(x.device != queries.device for x in (
        prefix_keys, prefix_values, current_keys, current_values, indices, head_to_kv
    )):
        raise RuntimeError("indexed-attention tensors must share a CUDA device")


def _partial(queries, prefix_keys, prefix_values, current_keys, current_values, indices,
             head_to_kv, valid_mask, split_tokens):
    """Batched core: queries [B, QH, D], prefix K/V [B, KVH, T, D] (strided), indices [B, QH, K]."""
    batch, q_heads, head_dim = (int(x) for x in queries.shape)
    kv_heads, prefix_tokens = int(prefix_keys.shape[1]), int(prefix_keys.shape[2])
    selected = int(indices.shape[-1])
    if prefix_tokens <= 0 or selected <= 0:
        raise ValueError("indexed attention requires non-empty prefix and selection")
    if prefix_keys.dtype != prefix_values.dtype or prefix_keys.dtype not in _lib.DTYPE_CODES:
        raise RuntimeError("prefix keys and values must share an fp32/fp16/bf16 dtype")
    if prefix_keys.stride(-1) != 1:
        prefix_keys = prefix_keys.contiguous()
    if prefix_values.stride(-1) != 1:
        prefix_values = prefix_values.contiguous()
    queries = queries.contiguous()
    current_keys = current_keys.to(prefix_keys.dtype).contiguous()
    current_values = current_values.to(prefix_keys.dtype).contiguous()
    if tuple(current_keys.shape) != (batch, kv_heads, head_dim) or current_values.shape != current_keys.shape:
        raise ValueError("current keys/values must be [KV heads, head dim]")
    indices = indices.to(torch.int64).contiguous()
    valid = None if valid_mask is None else valid_mask.to(torch.uint8).contiguous()
    mapping = head_to_kv.to(device=queries.device, dtype=torch.int64).contiguous()
    num_splits = math.ceil(selected / split_tokens)
    partials = torch.empty((batch, q_heads, num_splits, head_dim + 2), device=queries.device,
                           dtype=torch.float32)
    with torch.cuda.device(queries.device):
        _lib.check(_lib.lib().popkv_attn_partial(
            _lib.ptr(queries), _lib.dtype_code(queries), batch, q_heads, head_dim,
            _lib.ptr(prefix_keys), _lib.ptr(prefix_values), _lib.dtype_code(prefix_keys), kv_heads,
            prefix_tokens, int(prefix_keys.stride(0)), int(prefix_keys.stride(1)),
            int(prefix_keys.stride(2)), int(prefix_values.stride(0)), int(prefix_values.stride(1)),
            int(prefix_values.stride(2)), _lib.ptr(current_keys), _lib.ptr(current_values),
            _lib.ptr(indices), selected, _lib.ptr(valid), _lib.ptr(mapping), int(split_tokens),
            _lib.ptr(partials), _lib.stream_of(queries.device)))
    return partials


def indexed_attention_split_partial(
    queries: torch.Tensor, prefix_keys: torch.Tensor, prefix_values: torch.Tensor,
    current_keys: torch.Tensor, current_values: torch.Tensor, indices: torch.Tensor,
    head_to_kv: torch.Tensor, valid_mask: torch.Tensor | None = None, *,
    split_tokens: int = 256,
) -> torch.Tensor:
    """Token-tiled online-softmax partial attention states [QH, splits, D + 2] (fp32)."""
    _check_common(queries, prefix_keys, prefix_values, current_keys, current_values, indices,
                  head_to_kv, valid_mask, split_tokens, batched=False)
    partials = _partial(queries[None], prefix_keys[None], prefix_values[None], current_keys[None],
                        current_values[None], indices[None], head_to_kv,
                        None if valid_mask is None else valid_mask[None], split_tokens)
    return partials[0]


def indexed_attention_split_partial_batched(
    queries, prefix_keys, prefix_values, current_keys, current_values, indices, head_to_kv,
    valid_mask=None, *, split_tokens: int = 256,
) -> torch.Tensor:
    """Batched partials: queries [B, QH, D], prefix K/V [B, KVH, T, D] -> [B, QH, splits, D + 2]."""
    _check_common(queries, prefix_keys, prefix_values, current_keys, current_values, indices,
                  head_to_kv, valid_mask, split_tokens, batched=True)
    return _partial(queries, prefix_keys, prefix_values, current_keys, current_values, indices,
                    head_to_kv, valid_mask, split_tokens)


def indexed_attention_split_merge(partials: torch.Tensor, output_like: torch.Tensor) -> torch.Tensor:
    """Merge split online-softmax states into one output per query head."""
    if partials.ndim != 3 or partials.dtype != torch.float32 or not partials.is_cuda:
        raise ValueError("partials must be CUDA float32 [query heads, splits, D+2]")
    if output_like.ndim != 2 or output_like.device != partials.device:
        raise ValueError("output_like must be [query heads, head dim] on the partial device")
    q_heads, num_splits, state_d = (int(x) for x in partials.shape)
    head_dim = int(output_like.shape[1])
    if int(output_like.shape[0]) != q_heads or state_d != head_dim + 2:
        raise ValueError("partial/output shape mismatch")
    return _merge(partials, output_like.dtype, (q_heads, head_dim))


def indexed_attention_split_merge_batched(partials: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Merge [B, QH, splits, D + 2] partials into [B, QH, D] of ``dtype``."""
    if partials.ndim != 4 or partials.dtype != torch.float32 or not partials.is_cuda:
        raise ValueError("partials must be CUDA float32 [batch, query heads, splits, D+2]")
    batch, q_heads, _, state_d = (int(x) for x in partials.shape)
    return _merge(partials, dtype, (batch, q_heads, state_d - 2))


def _merge(partials: torch.Tensor, dtype: torch.dtype, out_shape) -> torch.Tensor:
    if dtype not in _lib.DTYPE_CODES:
        raise RuntimeError("output must be fp32/fp16/bf16")
    partials = partials.contiguous()
    num_splits, state_d = int(partials.shape[-2]), int(partials.shape[-1])
    rows = partials.numel() // (num_splits * state_d)
    output = torch.empty(out_shape, device=partials.device, dtype=dtype)
    with torch.cuda.device(partials.device):
        _lib.check(_lib.lib().popkv_attn_merge(
            _lib.ptr(partials), rows, num_splits, state_d - 2, _lib.ptr(output),
            _lib.dtype_code(output), _lib.stream_of(partials.device)))
    return output


def indexed_attention_split(
    queries: torch.Tensor, prefix_keys: torch.Tensor, prefix_values: torch.Tensor,
    current_keys: torch.Tensor, current_values: torch.Tensor, indices: torch.Tensor,
    head_to_kv: torch.Tensor, valid_mask: torch.Tensor | None = None, *,
    split_tokens: int = 256,
) -> torch.Tensor:
    """Split-token fused indexed attention with online-softmax merging."""
    partials = indexed_attention_split_partial(
        queries, prefix_keys, prefix_values, current_keys, current_values,
        indices, head_to_kv, valid_mask, split_tokens=split_tokens,
    )
    return indexed_attention_split_merge(partials, queries)


def indexed_attention(
    queries: torch.Tensor, prefix_keys: torch.Tensor, prefix_values: torch.Tensor,
    current_keys: torch.Tensor, current_values: torch.Tensor, indices: torch.Tensor,
    head_to_kv: torch.Tensor, valid_mask: torch.Tensor | None = None,
) -> torch.Tensor:
    """Unsplit indexed attention (reference sparse_kernels.py:105-233): one split per head."""
    selected = max(16, int(indices.shape[-1]))
    split = ((selected + 15) // 16) * 16
    return indexed_attention_split(queries, prefix_keys, prefix_values, current_keys,
                                   current_values, indices, head_to_kv, valid_mask,
                                   split_tokens=split)


def _outside_scope(name: str):
    def raiser(*args, **kwargs):
        raise NotImplementedError(
            f"{name} belongs to the QUEST comparison method, which popkv_b200 does not implement")
    raiser.__name__ = name
    return raiser


quest_scores = _outside_scope("quest_scores")
quest_indices = _outside_scope("quest_indices")
