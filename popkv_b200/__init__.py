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
import sys

from . import popkv, popkv_cuda, sparse_kernels  # noqa: F401
from ._lib import library_path  # noqa: F401

__all__ = ["popkv", "popkv_cuda", "sparse_kernels", "library_path", "install_as_reference_modules"]


def install_as_reference_modules() -> None:
    """Register this package's modules under the reference's top-level names.

    The reference imports its kernels lazily by module name
    (``from popkv_cuda import pack_keys`` at popkv.py:419, ``pack_keys_into``
    at :441 and :926, ``query_encode, score_encoded`` at :1078, and the split
    attention from ``sparse_kernels`` at :1106).  After this call those imports
    resolve to ``popkv_b200.popkv_cuda`` and ``popkv_b200.sparse_kernels``.
    Raises if a different ``popkv_cuda`` / ``sparse_kernels`` is already
    imported, since its functions may already be bound elsewhere.
    """
    for name, module in (("popkv_cuda", popkv_cuda), ("sparse_kernels", sparse_kernels)):
        present = sys.modules.get(name)
        if present is not None and present is not module:
            raise RuntimeError(f"module {name!r} is already imported from {getattr(present, '__file__', '?')}")
        sys.modules[name] = module
