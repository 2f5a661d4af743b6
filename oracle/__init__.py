"""CPU oracle for PopKV's decode-time retrieval path.

TEST INFRASTRUCTURE ONLY.  ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline legs of ``bench.py`` use this package as the checker; the product
(``popkv_b200``) never imports it.

The arithmetic lives in ``popkv_oracle.c`` (a C restatement of the reference's
kernels, each function citing the reference file:line it follows); this module
is the numpy/ctypes front end.  Element dtypes are given as strings: ``"f32"``
(np.float32 data), ``"f16"`` and ``"bf16"`` (raw 16-bit patterns in np.uint16).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

os.environ.setdefault("OMP_WAIT_POLICY", "PASSIVE")

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "build" / "libpopkv_oracle.so"
_DTYPES = {"f32": 0, "f16": 1, "bf16": 2}
_lib = None

_i64 = ctypes.c_int64
_ptr = ctypes.c_void_p


def build() -> Path:
    """Compile the C oracle with the committed Makefile (gcc, OpenMP)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        handle = ctypes.CDLL(str(_LIB_PATH))
        handle.oracle_pack.restype = ctypes.c_int
        handle.oracle_query_encode.restype = ctypes.c_int
        handle.oracle_score.restype = ctypes.c_int
        handle.oracle_topk.restype = ctypes.c_int
        handle.oracle_attn_partial.restype = ctypes.c_int
        handle.oracle_attn_merge.restype = ctypes.c_int
        handle.oracle_score_scale.restype = ctypes.c_float
        handle.oracle_score_scale.argtypes = [_i64]
        handle.oracle_float_to_half.restype = ctypes.c_uint16
        handle.oracle_float_to_half.argtypes = [ctypes.c_float]
        handle.oracle_half_to_float.restype = ctypes.c_float
        handle.oracle_half_to_float.argtypes = [ctypes.c_uint16]
        handle.oracle_num_threads.restype = ctypes.c_int
        _lib = handle
    return _lib


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def _p(array: np.ndarray | None):
    if array is None:
        return None
    assert array.flags["C_CONTIGUOUS"] or array.flags["WRITEABLE"]
    return array.ctypes.data_as(_ptr)


def _check(status: int, name: str) -> None:
    if status != 0:
        raise ValueError(f"oracle {name} rejected its arguments (status {status})")


def _elements(array: np.ndarray, dtype: str) -> np.ndarray:
    want = np.float32 if dtype == "f32" else np.uint16
    if array.dtype != want:
        raise TypeError(f"{dtype} data must be {want.__name__}, got {array.dtype}")
    return array


def words_for(head_dim: int) -> int:
    return (head_dim + 31) // 32


def reps_for(head_dim: int, dim_group_size: int) -> int:
    return (head_dim + dim_group_size - 1) // dim_group_size


def half_bits_to_float(bits: np.ndarray) -> np.ndarray:
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def to_float(array: np.ndarray, dtype: str) -> np.ndarray:
    """Exact float32 values of f32 / f16-bits / bf16-bits data."""
    if dtype == "f32":
        return np.asarray(array, dtype=np.float32)
    if dtype == "f16":
        return half_bits_to_float(array)
    return (np.asarray(array, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def score_scale(head_dim: int) -> float:
    return float(lib().oracle_score_scale(int(head_dim)))


def pack(keys: np.ndarray, dtype: str, *, token_group_size: int, dim_group_size: int,
         token_capacity: int | None = None, token_offset: int = 0, out=None):
    """Key bit-planes and representatives (popkv_cuda.py:53 / :72).

    ``keys`` is [kv_heads, tokens, head_dim] (any strides).  Returns or fills
    (k_sign int32, k_mag int32, k_low fp16 bits, k_delta fp16 bits), each
    [kv_heads, capacity, words|reps].
    """
    keys = _elements(keys, dtype)
    kv_heads, tokens, head_dim = keys.shape
    item = keys.itemsize
    head_stride, token_stride, dim_stride = (s // item for s in keys.strides)
    if dim_stride != 1:
        keys = np.ascontiguousarray(keys)
        head_stride, token_stride, _ = (s // item for s in keys.strides)
    words, reps = words_for(head_dim), reps_for(head_dim, dim_group_size)
    if out is None:
        capacity = tokens if token_capacity is None else int(token_capacity)
        out = (np.zeros((kv_heads, capacity, words), np.int32),
               np.zeros((kv_heads, capacity, words), np.int32),
               np.zeros((kv_heads, capacity, reps), np.uint16),
               np.zeros((kv_heads, capacity, reps), np.uint16))
    capacity = out[0].shape[1]
    status = lib().oracle_pack(
        _p(keys), _DTYPES[dtype], _i64(kv_heads), _i64(tokens), _i64(head_dim),
        _i64(head_stride), _i64(token_stride), _i64(token_group_size), _i64(dim_group_size),
        _i64(capacity), _i64(token_offset), _p(out[0]), _p(out[1]), _p(out[2]), _p(out[3]))
    _check(status, "pack")
    return out


def query_encode(queries: np.ndarray, dtype: str, *, dim_group_size: int):
    """(q_sign int32, q_mag int32, q_low f32, q_delta f32) of [B, QH, D] queries."""
    queries = np.ascontiguousarray(_elements(queries, dtype))
    batch, q_heads, head_dim = queries.shape
    words, reps = words_for(head_dim), reps_for(head_dim, dim_group_size)
    out = (np.zeros((batch, q_heads, words), np.int32), np.zeros((batch, q_heads, words), np.int32),
           np.zeros((batch, q_heads, reps), np.float32), np.zeros((batch, q_heads, reps), np.float32))
    status = lib().oracle_query_encode(
        _p(queries), _DTYPES[dtype], _i64(batch * q_heads), _i64(head_dim), _i64(dim_group_size),
        _p(out[0]), _p(out[1]), _p(out[2]), _p(out[3]))
    _check(status, "query_encode")
    return out


def score(encoded, packed, *, head_to_kv: np.ndarray, tokens: int, dim_group_size: int,
          head_dim: int):
    """Popcount scores: returns (fp32 [B,QH,tokens], fp16 bits [B,QH,tokens])."""
    q_sign, q_mag, q_low, q_delta = (np.ascontiguousarray(x) for x in encoded)
    k_sign, k_mag, k_low, k_delta = (np.ascontiguousarray(x) for x in packed)
    batch, q_heads, _ = q_sign.shape
    kv_heads, capacity, _ = k_sign.shape
    mapping = np.ascontiguousarray(head_to_kv, dtype=np.int64)
    out32 = np.zeros((batch, q_heads, tokens), np.float32)
    out16 = np.zeros((batch, q_heads, tokens), np.uint16)
    status = lib().oracle_score(
        _p(q_sign), _p(q_mag), _p(q_low), _p(q_delta), _i64(batch), _i64(q_heads),
        _p(k_sign), _p(k_mag), _p(k_low), _p(k_delta), _i64(kv_heads), _i64(capacity),
        _i64(head_dim), _i64(dim_group_size), _p(mapping), _i64(tokens), _p(out32), _p(out16))
    _check(status, "score")
    return out32, out16


def topk(scores: np.ndarray, k: int) -> np.ndarray:
    """Deterministic top-k over the last axis; ascending token indices, int64.

    ``scores`` is fp16 bits (np.uint16) or np.float32, shape [..., tokens].
    """
    is_f32 = scores.dtype == np.float32
    if not is_f32 and scores.dtype != np.uint16:
        raise TypeError("scores must be fp16 bits (uint16) or float32")
    lead = scores.shape[:-1]
    tokens = scores.shape[-1]
    flat = np.ascontiguousarray(scores).reshape(-1, tokens)
    out = np.zeros((flat.shape[0], k), np.int64)
    status = lib().oracle_topk(_p(flat), ctypes.c_int(int(is_f32)), _i64(flat.shape[0]),
                               _i64(tokens), _i64(tokens), _i64(k), _p(out), _i64(k))
    _check(status, "topk")
    return out.reshape(*lead, k)


def select_with_current(scores: np.ndarray, budget: int, prefix_tokens: int) -> np.ndarray:
    """top-(min(budget-1, prefix)) indices plus the current slot (popkv.py:1094-1098, :287-291)."""
    k = min(budget - 1, prefix_tokens)
    chosen = topk(scores[..., :prefix_tokens], k)
    current = np.full((*chosen.shape[:-1], 1), prefix_tokens, np.int64)
    return np.concatenate([chosen, current], axis=-1)


def attn_partial(queries, q_dtype, prefix_keys, prefix_values, kv_dtype, current_keys,
                 current_values, indices, head_to_kv, valid=None, *, split_tokens=256):
    """Partial states [QH, splits, D+2] in float64 (sparse_kernels.py:237-294)."""
    queries = np.ascontiguousarray(_elements(queries, q_dtype))
    q_heads, head_dim = queries.shape
    prefix_keys = _elements(prefix_keys, kv_dtype)
    prefix_values = _elements(prefix_values, kv_dtype)
    item = prefix_keys.itemsize
    if prefix_keys.strides[2] != item:
        prefix_keys = np.ascontiguousarray(prefix_keys)
    if prefix_values.strides[2] != item:
        prefix_values = np.ascontiguousarray(prefix_values)
    k_hs, k_ts = prefix_keys.strides[0] // item, prefix_keys.strides[1] // item
    v_hs, v_ts = prefix_values.strides[0] // item, prefix_values.strides[1] // item
    prefix_tokens = prefix_keys.shape[1]
    current_keys = np.ascontiguousarray(_elements(current_keys, kv_dtype))
    current_values = np.ascontiguousarray(_elements(current_values, kv_dtype))
    indices = np.ascontiguousarray(indices, dtype=np.int64)
    selected = indices.shape[1]
    valid_u8 = None if valid is None else np.ascontiguousarray(valid, dtype=np.uint8)
    mapping = np.ascontiguousarray(head_to_kv, dtype=np.int64)
    splits = (selected + split_tokens - 1) // split_tokens
    out = np.zeros((q_heads, splits, head_dim + 2), np.float64)
    status = lib().oracle_attn_partial(
        _p(queries), ctypes.c_int(_DTYPES[q_dtype]), _i64(q_heads), _i64(head_dim),
        _p(prefix_keys), _p(prefix_values), ctypes.c_int(_DTYPES[kv_dtype]), _i64(prefix_tokens),
        _i64(k_hs), _i64(k_ts), _i64(v_hs), _i64(v_ts), _p(current_keys), _p(current_values),
        _p(indices), _i64(selected), _p(valid_u8), _p(mapping), _i64(split_tokens), _p(out))
    _check(status, "attn_partial")
    return out


def attn_merge(partials: np.ndarray) -> np.ndarray:
    partials = np.ascontiguousarray(partials, dtype=np.float64)
    q_heads, splits, state = partials.shape
    out = np.zeros((q_heads, state - 2), np.float64)
    status = lib().oracle_attn_merge(_p(partials), _i64(q_heads), _i64(splits),
                                     _i64(state - 2), _p(out))
    _check(status, "attn_merge")
    return out


def attention(queries, q_dtype, prefix_keys, prefix_values, kv_dtype, current_keys,
              current_values, indices, head_to_kv, valid=None, *, split_tokens=256):
    return attn_merge(attn_partial(queries, q_dtype, prefix_keys, prefix_values, kv_dtype,
                                   current_keys, current_values, indices, head_to_kv, valid,
                                   split_tokens=split_tokens))


__all__ = [
    "build", "lib", "num_threads", "pack", "query_encode", "score", "score_scale", "topk",
    "select_with_current", "attn_partial", "attn_merge", "attention", "to_float",
    "half_bits_to_float", "words_for", "reps_for",
]
