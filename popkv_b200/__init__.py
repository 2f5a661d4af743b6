"""PopKV decode-time KV retrieval on NVIDIA B200 (sm_100a).

Drop-in for the reference's retrieval path:

* ``popkv_b200.popkv_cuda``     -- pack_keys, pack_keys_into, query_encode,
                                    allocate_query_encode_outputs, score_encoded,
                                    score, topk  (reference popkv_cuda.py)
* ``popkv_b200.sparse_kernels`` -- indexed_attention_split_partial / _merge /
                                    indexed_attention_split (+ batched forms)
                                    (reference sparse_kernels.py)
* ``popkv_b200.popkv``          -- RetrievalConfig, POPKV_PRESETS, PopKVCache,
                                    build_popkv_cache, append_popkv, _append_current,
                                    popkv_attention (reference popkv.py)
* ``popkv_b200.sharding``       -- KV-head sharding across GPUs with one
                                    all-gather of head outputs per layer

All compute runs in ``lib/libpopkv_b200.so`` (hand-written CUDA for sm_100a
behind the C ABI in ``include/popkv_b200.h``).
"""
from . import popkv, popkv_cuda, sparse_kernels  # noqa: F401
from ._lib import library_path  # noqa: F401

__all__ = ["popkv", "popkv_cuda", "sparse_kernels", "library_path"]
