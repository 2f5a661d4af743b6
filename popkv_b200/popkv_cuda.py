"""Drop-in replacement of the reference's ``popkv_cuda`` op wrappers (popkv_cuda.py).

Same functions, argument names, shapes, dtypes and error behaviour as the
reference module: argument validation raises ``ValueError`` with the reference's
messages, and failures inside the native library raise ``RuntimeError`` (the
reference's TORCH_CHECK errors).  Every op runs the sm_100a kernels of
``libpopkv_b200.so`` on the current CUDA stream of the input's device.

Differences a caller can observe:
* key representatives and query low/delta use correctly rounded division (the
  reference builds with --use_fast_math), so a value can differ from the
  reference's by one rounding step; sign/magnitude planes are identical;
* ``score`` and ``score_encoded`` share one query encoder, so they agree bit
  for bit for every input (the reference's two paths encode with different
  summation orders);
* QUEST and FIER helpers are outside this package and raise NotImplementedError.
"""
from __future__ import annotations

import torch

from . import _lib

MAX_TOKEN_GROUP_SIZE = 4096
SPECIALIZED_TOKEN_GROUP_SIZES = (8, 16, 32, 64, 128)
SUPPORTED_DIM_KERNELS = ("g16", "g32", "g64-u32", "g64-u64")


def _validate_token_group_size(token_group_size: int) -> int:
    value = int(token_group_size)
    if not 1 <= value <= MAX_TOKEN_GROUP_SIZE:
        raise ValueError(f"token_group_size must be between 1 and {MAX_TOKEN_GROUP_SIZE}")
    return value


def _validate_dim_group_size(dim_group_size: int) -> int:
    value = int(dim_group_size)
    if value not in (16, 32, 64):
        raise ValueError("dim_group_size must be one of 16, 32, 64")
    return value


def _validate_dim_kernel(dim_group_size: int, dim_kernel: str | None) -> str:
    default = {16: "g16", 32: "g32", 64: "g64-u32"}[dim_group_size]
    value = default if dim_kernel is None or dim_kernel == "auto" else str(dim_kernel)
    if value not in SUPPORTED_DIM_KERNELS:
        raise ValueError(f"dim_kernel must be one of {SUPPORTED_DIM_KERNELS}")
    expected = 64 if value.startswith("g64-") else int(value[1:])
    if expected != dim_group_size:
        raise ValueError(f"dim_kernel={value} requires dim_group_size={expected}")
    return value


def _check_keys(keys: torch.Tensor) -> None:
    if keys.ndim != 3 or not keys.is_cuda or not keys.is_contiguous():
        raise ValueError("keys must be contiguous CUDA [KV heads, tokens, head dim]")


def _check_group_combo(token_group_size: int, dim_group_size: int) -> None:
    if dim_group_size != 32 and token_group_size not in SPECIALIZED_TOKEN_GROUP_SIZES:
        raise ValueError("non-specialized token group sizes require dim_group_size=32")


def _require(condition: bool, message: str) -> None:
    if not condition:
        raise RuntimeError(message)


def _check_planes(packed, kv_heads: int, head_dim: int, dim_group_size: int, device) -> int:
    k_sign, k_mag, k_low, k_delta = packed
    words = (head_dim + 31) // 32
    reps = (head_dim + dim_group_size - 1) // dim_group_size
    for tensor in packed:
        _require(tensor.is_cuda, "packed planes must be CUDA tensors")
        _require(tensor.is_contiguous(), "packed planes must be contiguous")
        _require(tensor.device == device, "Pop-KV packing tensors must share a CUDA device")
    _require(k_sign.dtype == torch.int32 and k_mag.dtype == torch.int32, "k_sign must be int32")
    _require(k_low.dtype == torch.float16 and k_delta.dtype == torch.float16,
             "Pop-KV representative metadata must be float16")
    _require(k_sign.ndim == 3 and k_sign.shape[0] == kv_heads and k_sign.shape[2] == words
             and k_mag.shape == k_sign.shape, "packed bitplane shape mismatch")
    _require(k_low.ndim == 3 and k_low.shape[0] == kv_heads and k_low.shape[1] == k_sign.shape[1]
             and k_low.shape[2] == reps and k_delta.shape == k_low.shape,
             "representative metadata shape mismatch")
    return int(k_sign.shape[1])


def _pack_launch(keys: torch.Tensor, packed, token_offset: int, token_group_size: int,
                 dim_group_size: int) -> None:
    kv_heads, tokens, head_dim = (int(x) for x in keys.shape)
    capacity = int(packed[0].shape[1])
    _require(keys.dtype in _lib.DTYPE_CODES, "keys must be fp32/fp16/bf16")
    _require(token_offset >= 0 and token_offset + tokens <= capacity, "Pop-KV cache capacity exceeded")
    with torch.cuda.device(keys.device):
        _lib.check(_lib.lib().popkv_pack(
            _lib.ptr(keys), _lib.dtype_code(keys), kv_heads, tokens, head_dim,
            int(keys.stride(0)), int(keys.stride(1)), *(_lib.ptr(t) for t in packed), capacity,
            int(token_offset), int(token_group_size), int(dim_group_size),
            _lib.stream_of(keys.device)))


def pack_keys(
    keys: torch.Tensor, *, token_capacity: int | None = None,
    token_group_size: int = 32, dim_group_size: int = 32,
):
    """Pack fixed uint32 K bitplanes plus G_dim low/delta representatives.

    Returns (k_sign int32, k_mag int32, k_low fp16, k_delta fp16), each
    [KV heads, capacity, words|reps]; rows past ``keys.shape[1]`` are left
    uninitialised, as in the reference (popkv_cuda.py:53-69).
    """
    _check_keys(keys)
    capacity = int(keys.shape[1]) if token_capacity is None else int(token_capacity)
    token_group_size = _validate_token_group_size(token_group_size)
    dim_group_size = _validate_dim_group_size(dim_group_size)
    _check_group_combo(token_group_size, dim_group_size)
    kv_heads, tokens, head_dim = (int(x) for x in keys.shape)
    _require(head_dim > 0, "keys must be [KVH, non-empty tokens, non-empty head dim]")
    _require(capacity >= tokens, "token capacity is too small")
    words = (head_dim + 31) // 32
    reps = (head_dim + dim_group_size - 1) // dim_group_size
    k_sign = torch.empty((kv_heads, capacity, words), device=keys.device, dtype=torch.int32)
    k_mag = torch.empty_like(k_sign)
    k_low = torch.empty((kv_heads, capacity, reps), device=keys.device, dtype=torch.float16)
    k_delta = torch.empty_like(k_low)
    packed = (k_sign, k_mag, k_low, k_delta)
    _pack_launch(keys, packed, 0, token_group_size, dim_group_size)
    return packed


def pack_keys_into(
    keys: torch.Tensor, packed, *, token_offset: int,
    token_group_size: int = 32, dim_group_size: int = 32,
) -> None:
    """Re-encode ``keys`` into rows [token_offset, token_offset + T) of ``packed``."""
    _check_keys(keys)
    token_group_size = _validate_token_group_size(token_group_size)
    dim_group_size = _validate_dim_group_size(dim_group_size)
    _check_group_combo(token_group_size, dim_group_size)
    packed = tuple(packed)
    _require(len(packed) == 4, "packed must contain k_sign, k_mag, k_low, k_delta")
    _check_planes(packed, int(keys.shape[0]), int(keys.shape[2]), dim_group_size, keys.device)
    _pack_launch(keys, packed, int(token_offset), token_group_size, dim_group_size)


def _outside_scope(name: str):
    def raiser(*args, **kwargs):
        raise NotImplementedError(
            f"{name} belongs to the QUEST/FIER comparison methods, which popkv_b200 does not "
            "implement; use the reference package for those baselines")
    raiser.__name__ = name
    return raiser


update_quest_metadata = _outside_scope("update_quest_metadata")
update_fier_legacy_metadata = _outside_scope("update_fier_legacy_metadata")
update_fier_metadata = _outside_scope("update_fier_metadata")
score_fier = _outside_scope("score_fier")


def allocate_query_encode_outputs(queries: torch.Tensor, *, dim_group_size: int = 32):
    """Allocate outputs matching the fused scorer's query state."""
    if queries.ndim != 3 or not queries.is_cuda or not queries.is_contiguous():
        raise ValueError("queries must be contiguous CUDA [batch, query heads, head dim]")
    words = (int(queries.shape[2]) + 31) // 32
    dim_group_size = _validate_dim_group_size(dim_group_size)
    groups = (int(queries.shape[2]) + dim_group_size - 1) // dim_group_size
    bit_shape = (int(queries.shape[0]), int(queries.shape[1]), words)
    rep_shape = (int(queries.shape[0]), int(queries.shape[1]), groups)
    sign = torch.empty(bit_shape, device=queries.device, dtype=torch.int32)
    magnitude = torch.empty_like(sign)
    low = torch.empty(rep_shape, device=queries.device, dtype=torch.float32)
    delta = torch.empty_like(low)
    return sign, magnitude, low, delta


def query_encode(queries: torch.Tensor, *, out=None, dim_group_size: int = 32):
    """Encode a PopKV query into bitplanes and dimension-group representatives."""
    if queries.ndim != 3 or not queries.is_cuda or not queries.is_contiguous():
        raise ValueError("queries must be contiguous CUDA [batch, query heads, head dim]")
    dim_group_size = _validate_dim_group_size(dim_group_size)
    outputs = (allocate_query_encode_outputs(queries, dim_group_size=dim_group_size)
               if out is None else tuple(out))
    if len(outputs) != 4:
        raise ValueError("out must contain q_sign, q_mag, q_low, q_delta")
    batch, q_heads, head_dim = (int(x) for x in queries.shape)
    _require(head_dim > 0, "queries must be [batch, query heads, non-empty head dim]")
    _require(queries.dtype in _lib.DTYPE_CODES, "queries must be fp32/fp16/bf16")
    words = (head_dim + 31) // 32
    reps = (head_dim + dim_group_size - 1) // dim_group_size
    q_sign, q_mag, q_low, q_delta = outputs
    for tensor in outputs:
        _require(tensor.is_cuda and tensor.is_contiguous(), "query encoding outputs must be contiguous CUDA")
        _require(tensor.device == queries.device, "query encoding tensors must share a CUDA device")
    _require(q_sign.dtype == torch.int32 and q_mag.dtype == torch.int32, "q_sign must be int32")
    _require(q_low.dtype == torch.float32 and q_delta.dtype == torch.float32,
             "query low/delta outputs must be float32")
    _require(tuple(q_sign.shape) == (batch, q_heads, words) and q_mag.shape == q_sign.shape
             and tuple(q_low.shape) == (batch, q_heads, reps) and q_delta.shape == q_low.shape,
             "query encoding outputs have incorrect shape")
    with torch.cuda.device(queries.device):
        _lib.check(_lib.lib().popkv_query_encode(
            _lib.ptr(queries), _lib.dtype_code(queries), batch * q_heads, head_dim, dim_group_size,
            *(_lib.ptr(t) for t in outputs), _lib.stream_of(queries.device)))
    return outputs


def _check_score_args(head_to_kv: torch.Tensor, q_heads: int, kv_heads: int, tokens: int,
                      capacity: int, device) -> torch.Tensor:
    _require(head_to_kv.dtype == torch.int64, "head mapping must be int64")
    _require(head_to_kv.is_cuda and head_to_kv.device == device, "score tensors must share a CUDA device")
    _require(head_to_kv.numel() == q_heads and q_heads % kv_heads == 0, "invalid GQA head mapping")
    _require(0 < tokens <= capacity, "invalid score token count")
    return head_to_kv.contiguous()


def score_encoded(
    encoded_query, packed, *, head_to_kv: torch.Tensor, tokens: int,
    dim_group_size: int = 32, dim_kernel: str | None = None,
) -> torch.Tensor:
    """Score compressed keys from a pre-encoded head-dim-128 PopKV query (fp16 out)."""
    dim_group_size = _validate_dim_group_size(dim_group_size)
    _validate_dim_kernel(dim_group_size, dim_kernel)
    encoded_query = tuple(encoded_query)
    packed = tuple(packed)
    if len(encoded_query) != 4:
        raise ValueError("encoded_query must contain q_sign, q_mag, q_low, q_delta")
    if len(packed) != 4:
        raise ValueError("packed must contain k_sign, k_mag, k_low, k_delta")
    if any(not tensor.is_cuda or not tensor.is_contiguous() for tensor in encoded_query):
        raise ValueError("encoded query tensors must be contiguous CUDA tensors")
    q_sign, q_mag, q_low, q_delta = encoded_query
    _require(q_sign.dtype == torch.int32 and q_mag.dtype == torch.int32, "q_sign must be int32")
    _require(q_low.dtype == torch.float32 and q_delta.dtype == torch.float32,
             "encoded Pop-KV query representatives must be float32")
    _require(q_sign.ndim == 3 and q_sign.shape[2] == 4 and q_mag.shape == q_sign.shape,
             "encoded Pop-KV query bitplanes must be [batch, query heads, 4]")
    batch, q_heads = int(q_sign.shape[0]), int(q_sign.shape[1])
    reps = 128 // dim_group_size
    _require(q_low.shape == q_delta.shape and q_low.ndim == 3 and tuple(q_low.shape) == (batch, q_heads, reps),
             "encoded Pop-KV query representative shape mismatch")
    device = q_sign.device
    kv_heads = int(packed[0].shape[0]) if packed[0].ndim == 3 else -1
    _require(packed[0].ndim == 3 and packed[0].shape[2] == 4 and packed[1].shape == packed[0].shape,
             "Pop-KV key bitplanes must be [KV heads, capacity, 4]")
    capacity = _check_planes(packed, kv_heads, 128, dim_group_size, device)
    for tensor in encoded_query:
        _require(tensor.device == device, "encoded score tensors must share a CUDA device")
    mapping = _check_score_args(head_to_kv, q_heads, kv_heads, int(tokens), capacity, device)
    scores = torch.empty((batch, q_heads, int(tokens)), device=device, dtype=torch.float16)
    with torch.cuda.device(device):
        _lib.check(_lib.lib().popkv_score_encoded(
            *(_lib.ptr(t) for t in encoded_query), batch, q_heads, *(_lib.ptr(t) for t in packed),
            kv_heads, capacity, _lib.ptr(mapping), int(tokens), dim_group_size, _lib.ptr(scores),
            _lib.stream_of(device)))
    return scores


_SCORE_DISPATCH = {"auto": 0, "popcount": 1, "fp8": 2}


def set_score_dispatch(mode: str) -> None:
    """Process-wide head_dim-128 scorer choice of every score entry point.

    ``"auto"`` (default): the fp8 tensor-core scorer from about one 128-token
    tile per SM up, the popcount scorer below; ``"popcount"``: always the
    popcount scorer; ``"fp8"``: the tensor-core scorer wherever it applies.
    The bits are the same; this is for tuning and testing.
    """
    if mode not in _SCORE_DISPATCH:
        raise ValueError("mode must be 'auto', 'popcount' or 'fp8'")
    _lib.check(_lib.lib().popkv_score_dispatch(_SCORE_DISPATCH[mode]))


def score(
    queries: torch.Tensor, packed, *, head_to_kv: torch.Tensor, tokens: int,
    dim_group_size: int = 32, dim_kernel: str | None = None, kernel: str = "auto",
) -> torch.Tensor:
    """Return approximate QK scores; the head-dim-128 fast path emits FP16, others FP32.

    ``kernel="auto"`` takes the library's choice for head_dim 128 (see
    ``set_score_dispatch``): the fp8 tensor-core scorer (tcgen05 e4m3 counts,
    at most 4 query heads per KV head) when the shape is large enough for it to
    win, the popcount scorer otherwise; ``"popcount"`` forces the popcount
    scorer and ``"tensor_core"`` forms the counts with tcgen05 int8 matrix
    products.  The scores are identical for all of them.
    """
    if kernel not in ("auto", "popcount", "tensor_core"):
        raise ValueError("kernel must be 'auto', 'popcount' or 'tensor_core'")
    if queries.ndim != 3 or not queries.is_cuda or not queries.is_contiguous():
        raise ValueError("queries must be contiguous CUDA [batch, query heads, head dim]")
    dim_group_size = _validate_dim_group_size(dim_group_size)
    _validate_dim_kernel(dim_group_size, dim_kernel)
    packed = tuple(packed)
    _require(len(packed) == 4, "packed must contain k_sign, k_mag, k_low, k_delta")
    _require(queries.dtype in _lib.DTYPE_CODES, "queries must be fp32/fp16/bf16")
    batch, q_heads, head_dim = (int(x) for x in queries.shape)
    kv_heads = int(packed[0].shape[0])
    capacity = _check_planes(packed, kv_heads, head_dim, dim_group_size, queries.device)
    mapping = _check_score_args(head_to_kv, q_heads, kv_heads, int(tokens), capacity, queries.device)
    out_dtype = torch.float16 if head_dim == 128 else torch.float32
    scores = torch.empty((batch, q_heads, int(tokens)), device=queries.device, dtype=out_dtype)
    with torch.cuda.device(queries.device):
        entry = {"auto": _lib.lib().popkv_score, "popcount": _lib.lib().popkv_score_popcount,
                 "tensor_core": _lib.lib().popkv_score_tc}[kernel]
        _lib.check(entry(
            _lib.ptr(queries), _lib.dtype_code(queries), batch, q_heads, head_dim,
            *(_lib.ptr(t) for t in packed), kv_heads, capacity, _lib.ptr(mapping), int(tokens),
            dim_group_size, _lib.ptr(scores), _lib.dtype_code(scores),
            _lib.stream_of(queries.device)))
    return scores


def topk(scores: torch.Tensor, k: int, *, current_index: int | None = None) -> torch.Tensor:
    """Deterministic top-k indices over the last axis of fp16/fp32 ``scores``.

    Returns int64 [..., k] (or [..., k + 1] with ``current_index`` appended), the
    k best tokens in ascending index order; ties rank by lower index.  Use as
    ``LlamaSparseDecoder.experimental_topk`` (reference popkv.py:1091-1093).
    """
    if not scores.is_cuda or scores.dtype not in (torch.float16, torch.float32):
        raise ValueError("scores must be a CUDA fp16/fp32 tensor")
    if scores.ndim < 1:
        raise ValueError("scores must have a token axis")
    tokens = int(scores.shape[-1])
    k = int(k)
    if not 0 <= k <= tokens:
        raise ValueError(f"k must be between 0 and {tokens}")
    if scores.stride(-1) != 1:
        scores = scores.contiguous()
    lead = tuple(scores.shape[:-1])
    flat = scores.reshape(-1, tokens) if scores.ndim > 1 else scores.reshape(1, tokens)
    if flat.ndim == 2 and flat.shape[0] > 1 and flat.stride(0) < tokens:
        flat = flat.contiguous()
    rows = int(flat.shape[0])
    width = k + (0 if current_index is None else 1)
    out = torch.empty((rows, width), device=scores.device, dtype=torch.int64)
    row_stride = int(flat.stride(0)) if rows > 1 else tokens
    with torch.cuda.device(scores.device):
        _lib.check(_lib.lib().popkv_topk(
            _lib.ptr(flat), _lib.dtype_code(flat), rows, tokens, row_stride, k,
            -1 if current_index is None else int(current_index), _lib.ptr(out), width,
            _lib.stream_of(scores.device)))
    return out.reshape(*lead, width)
