"""PopKV retrieval state and the per-layer sparse decode step.

Mirrors the PopKV parts of the reference's method layer (popkv.py): the
``RetrievalConfig`` / ``POPKV_PRESETS`` configuration (popkv.py:20-64), the
``PopKVCache`` state with ``build_popkv_cache`` / ``append_popkv``
(popkv.py:89-96, :416-459), current-slot reservation (popkv.py:287-291), and
the decoder's PopKV branch (popkv.py:1076-1115) as ``popkv_attention``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib, popkv_cuda, sparse_kernels

METHODS = ("popkv-normal", "popkv-q", "popkv-s")
POPKV_PRESETS = {
    "popkv-normal": (32, 32),
    "popkv-q": (128, 16),
    "popkv-s": (64, 64),
}
TOKEN_GROUP_SIZE = 32
SPECIALIZED_TOKEN_GROUP_SIZES = (8, 16, 32, 64, 128)
MAX_TOKEN_GROUP_SIZE = 4096
SUPPORTED_TOKEN_GROUP_SIZES = SPECIALIZED_TOKEN_GROUP_SIZES
PACKING_WORD_BITS = 32
SUPPORTED_DIM_GROUP_SIZES = (16, 32, 64)
SUPPORTED_DIM_KERNELS = ("auto", "g16", "g32", "g64-u32", "g64-u64")


@dataclass(frozen=True)
class RetrievalConfig:
    budget: int = 4096
    group_size: int = 32  # token-axis magnitude-threshold group (B_token)
    dim_group_size: int = 32  # dimensions sharing low/delta representatives (G_dim)
    dim_kernel: str = "auto"  # specialized score kernel; auto follows G_dim
    quest_page_size: int = 16
    fier_kernel: str = "fier"
    full_layers: tuple[int, ...] = (0, 1)

    def validate(self) -> None:
        if self.budget <= 1:
            raise ValueError("budget must reserve at least one retrieved and one current token")
        if not 1 <= self.group_size <= MAX_TOKEN_GROUP_SIZE:
            raise ValueError(f"group_size must be between 1 and {MAX_TOKEN_GROUP_SIZE}")
        if self.dim_group_size != 32 and self.group_size not in SPECIALIZED_TOKEN_GROUP_SIZES:
            raise ValueError("non-specialized token group sizes require dim_group_size=32")
        if self.dim_group_size not in SUPPORTED_DIM_GROUP_SIZES:
            raise ValueError("dim_group_size must be one of 16, 32, 64")
        if self.dim_kernel not in SUPPORTED_DIM_KERNELS:
            raise ValueError(f"dim_kernel must be one of {SUPPORTED_DIM_KERNELS}")
        if self.dim_kernel != "auto":
            expected = 64 if self.dim_kernel.startswith("g64-") else int(self.dim_kernel[1:])
            if expected != self.dim_group_size:
                raise ValueError(
                    f"dim_kernel={self.dim_kernel} requires dim_group_size={expected}"
                )
        if self.quest_page_size <= 0:
            raise ValueError("quest_page_size must be positive")
        if self.fier_kernel != "fier":
            raise ValueError("the public FIER method is fixed to the FIER implementation")


@dataclass
class PopKVCache:
    group_size: int
    dim_group_size: int
    token_count: int
    sealed_tokens: int
    packed: tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]
    active_keys: torch.Tensor


def _sparse_layer_indices(num_layers: int, full_layers) -> tuple[int, ...]:
    return tuple(layer for layer in range(num_layers) if layer not in full_layers)


def _append_current(indices: torch.Tensor, num_tokens: int) -> torch.Tensor:
    """Reserve the last slot for the current token, index ``num_tokens - 1`` (popkv.py:287-291)."""
    current = torch.full(
        (*indices.shape[:-1], 1), num_tokens - 1, device=indices.device, dtype=torch.long,
    )
    return torch.cat([indices.long(), current], dim=-1)


def build_popkv_cache(
    keys: torch.Tensor, *, group_size: int, dim_group_size: int = 32, reserve_tokens: int,
) -> PopKVCache:
    """Prepack the prefix keys [KVH, T, D] (popkv.py:416-435)."""
    if not 1 <= group_size <= MAX_TOKEN_GROUP_SIZE:
        raise ValueError(f"Pop-KV group_size must be between 1 and {MAX_TOKEN_GROUP_SIZE}")
    if dim_group_size != 32 and group_size not in SPECIALIZED_TOKEN_GROUP_SIZES:
        raise ValueError("non-specialized token group sizes require dim_group_size=32")
    if dim_group_size not in (16, 32, 64):
        raise ValueError("dim_group_size must be one of 16, 32, 64")
    tokens = int(keys.shape[1])
    capacity = math.ceil((tokens + reserve_tokens) / group_size) * group_size
    packed = popkv_cuda.pack_keys(keys.contiguous(), token_capacity=capacity,
                                  token_group_size=group_size, dim_group_size=dim_group_size)
    sealed = (tokens // group_size) * group_size
    return PopKVCache(
        group_size, dim_group_size, tokens, sealed, packed,
        keys[:, sealed:].detach().clone().contiguous(),
    )


def append_popkv(cache: PopKVCache, keys: torch.Tensor, timer=None) -> None:
    """Append one token's keys [KVH, 1, D] and re-encode the active group (popkv.py:438-459)."""
    cache.active_keys = torch.cat([cache.active_keys, keys.detach()], dim=1).contiguous()
    if timer: timer.mark("active_key_staging")
    if cache.sealed_tokens + int(cache.active_keys.shape[1]) > int(cache.packed[0].shape[1]):
        raise RuntimeError("Pop-KV cache reserve exhausted")
    popkv_cuda.pack_keys_into(
        cache.active_keys, cache.packed, token_offset=cache.sealed_tokens,
        token_group_size=cache.group_size,
        dim_group_size=cache.dim_group_size,
    )
    if timer:
        timer.mark("k_metadata_encoding")
        timer.mark("metadata_write")  # Stores are fused into the encoding kernel.
    cache.token_count += 1
    if int(cache.active_keys.shape[1]) == cache.group_size:
        cache.sealed_tokens += cache.group_size
        cache.active_keys = cache.active_keys[:, :0].contiguous()
    if timer: timer.mark("group_sealing")


def append_popkv_kv(cache: PopKVCache, key_cache: torch.Tensor, value_cache: torch.Tensor,
                    new_keys: torch.Tensor, new_values: torch.Tensor) -> None:
    """Append one decoded token to the static K/V caches and re-encode its group, in one launch.

    ``key_cache`` / ``value_cache`` [KVH, T, 128] (strided views allowed, head
    dim contiguous) hold the cached tokens; the new token goes to row
    ``cache.token_count``.  Unlike :func:`append_popkv` (popkv.py:438-459) no
    ``active_keys`` copy is staged: the open group is re-encoded straight from
    the key cache (popkv_append_kv).  ``cache.active_keys`` becomes a view of the
    open group's rows.
    """
    from . import _lib
    if key_cache.ndim != 3 or value_cache.ndim != 3 or key_cache.stride(-1) != 1 or value_cache.stride(-1) != 1:
        raise ValueError("key/value caches must be [KV heads, tokens, head dim] with a contiguous head dim")
    kv_heads, rows, head_dim = (int(x) for x in key_cache.shape)
    position = cache.token_count
    if position >= rows or position >= int(cache.packed[0].shape[1]):
        raise RuntimeError("Pop-KV cache reserve exhausted")
    nk = new_keys.reshape(kv_heads, head_dim).to(key_cache.dtype).contiguous()
    nv = new_values.reshape(kv_heads, head_dim).to(value_cache.dtype).contiguous()
    with torch.cuda.device(key_cache.device):
        _lib.check(_lib.lib().popkv_append_kv(
            _lib.ptr(nk), _lib.ptr(nv), _lib.dtype_code(key_cache), kv_heads, head_dim, _lib.ptr(key_cache),
            _lib.ptr(value_cache), key_cache.stride(0), key_cache.stride(1), value_cache.stride(0),
            value_cache.stride(1), position, *(_lib.ptr(t) for t in cache.packed),
            int(cache.packed[0].shape[1]), cache.sealed_tokens, cache.group_size, cache.dim_group_size,
            _lib.stream_of(key_cache.device)))
    cache.token_count += 1
    if cache.token_count - cache.sealed_tokens == cache.group_size:
        cache.sealed_tokens += cache.group_size
    cache.active_keys = key_cache[:, cache.sealed_tokens:cache.token_count]


def topk(scores: torch.Tensor, k: int) -> torch.Tensor:
    """Deterministic replacement of torch.topk(scores, k, sorted=False).indices.

    Ties rank by lower token index; winners come back in ascending index order.
    Drop-in for ``LlamaSparseDecoder.experimental_topk`` (popkv.py:1091-1093).
    """
    return popkv_cuda.topk(scores, k)


def select_tokens(scores: torch.Tensor, *, budget: int, prefix_tokens: int) -> torch.Tensor:
    """top-(budget-1) over the first ``prefix_tokens`` scores plus the current slot.

    ``scores`` is [B, QH, >= prefix_tokens]; returns int64 [B, QH, min(budget-1,
    prefix) + 1] whose last column is ``prefix_tokens`` (popkv.py:1090-1099).
    """
    k = min(int(budget) - 1, int(prefix_tokens))
    return popkv_cuda.topk(scores[..., :prefix_tokens], k, current_index=int(prefix_tokens))


def popkv_attention(
    queries: torch.Tensor, prefix_keys: torch.Tensor, prefix_values: torch.Tensor,
    current_keys: torch.Tensor, current_values: torch.Tensor, cache: PopKVCache,
    head_to_kv: torch.Tensor, *, budget: int, split_tokens: int = 256,
) -> torch.Tensor:
    """One layer's PopKV branch (popkv.py:1076-1115) for batch 1.

    queries [QH, D]; prefix_keys/values [KVH, prefix, D] (strided views are fine);
    current_keys/values [KVH, D].  Returns [QH, D] in the queries' dtype.
    """
    prefix_tokens = int(prefix_keys.shape[1])
    encoded = popkv_cuda.query_encode(queries.unsqueeze(0).contiguous(),
                                      dim_group_size=cache.dim_group_size)
    scores = popkv_cuda.score_encoded(
        encoded, cache.packed, head_to_kv=head_to_kv, tokens=cache.token_count,
        dim_group_size=cache.dim_group_size,
    )
    indices = select_tokens(scores, budget=budget, prefix_tokens=prefix_tokens)[0]
    partials = sparse_kernels.indexed_attention_split_partial(
        queries, prefix_keys, prefix_values, current_keys, current_values, indices, head_to_kv,
        None, split_tokens=split_tokens,
    )
    return sparse_kernels.indexed_attention_split_merge(partials, queries)


def popkv_retrieve(
    queries: torch.Tensor, packed, prefix_keys: torch.Tensor, prefix_values: torch.Tensor,
    current_keys: torch.Tensor, current_values: torch.Tensor, head_to_kv: torch.Tensor, *,
    tokens: int, budget: int, dim_group_size: int, out: torch.Tensor | None = None,
    return_scores: bool = False, return_indices: bool = False,
):
    """The whole PopKV decode branch (popkv.py:1076-1115) in one fused launch.

    queries [B, QH, 128]; packed planes [KVH, cap, *] (B == 1) or
    [B, KVH, cap, *]; prefix K/V [B, KVH, T, 128] or [KVH, T, 128] (strided
    views allowed); current K/V [B, KVH, 128] or [KVH, 128].  Scores the first
    ``tokens`` cached keys, keeps the top ``min(budget - 1, tokens)`` per query
    head plus the current slot, and returns the attention output [B, QH, 128]
    -- the same selection as score -> topk -> split attention.  With
    ``return_scores`` / ``return_indices`` also returns the fp16 scores and the
    int64 selected indices (last column = current slot).
    """
    if queries.ndim != 3 or not queries.is_cuda:
        raise ValueError("queries must be CUDA [batch, query heads, head dim]")
    batch, q_heads, head_dim = (int(x) for x in queries.shape)
    if prefix_keys.ndim == 3:
        prefix_keys, prefix_values = prefix_keys[None], prefix_values[None]
    if current_keys.ndim == 2:
        current_keys, current_values = current_keys[None], current_values[None]
    packed = tuple(packed)
    if len(packed) != 4:
        raise ValueError("packed must contain k_sign, k_mag, k_low, k_delta")
    if packed[0].ndim == 3:
        if batch != 1:
            raise ValueError("batched retrieval needs planes stacked as [batch, KV heads, capacity, *]")
        kv_heads, capacity = int(packed[0].shape[0]), int(packed[0].shape[1])
        plane_batch_stride = kv_heads * capacity
    else:
        kv_heads, capacity = int(packed[0].shape[1]), int(packed[0].shape[2])
        plane_batch_stride = kv_heads * capacity
    for t in packed:
        if not t.is_contiguous():
            raise ValueError("packed planes must be contiguous")
    queries = queries.contiguous()
    current_keys = current_keys.to(prefix_keys.dtype).contiguous()
    current_values = current_values.to(prefix_keys.dtype).contiguous()
    mapping = head_to_kv.to(device=queries.device, dtype=torch.int64).contiguous()
    if out is None:
        out = torch.empty_like(queries)
    k = min(int(budget) - 1, int(tokens))
    scores = (torch.empty((batch, q_heads, int(tokens)), device=queries.device, dtype=torch.float16)
              if return_scores else None)
    indices = (torch.empty((batch, q_heads, k + 1), device=queries.device, dtype=torch.int64)
               if return_indices else None)
    with torch.cuda.device(queries.device):
        _lib.check(_lib.lib().popkv_retrieve(
            _lib.ptr(queries), _lib.dtype_code(queries), batch, q_heads, head_dim,
            *(_lib.ptr(t) for t in packed), kv_heads, capacity, plane_batch_stride, int(tokens),
            int(dim_group_size), _lib.ptr(mapping), _lib.ptr(prefix_keys), _lib.ptr(prefix_values),
            _lib.dtype_code(prefix_keys), prefix_keys.stride(0), prefix_keys.stride(1),
            prefix_keys.stride(2), prefix_values.stride(0), prefix_values.stride(1),
            prefix_values.stride(2), _lib.ptr(current_keys), _lib.ptr(current_values), int(budget),
            _lib.ptr(out), _lib.ptr(scores), _lib.ptr(indices), _lib.stream_of(queries.device)))
    if return_scores or return_indices:
        return out, scores, indices
    return out
