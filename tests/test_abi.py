"""The C-ABI library loads, exports every declared symbol, and validates on the host.

No test here launches a kernel: argument validation happens before any CUDA
call, so these run without a GPU.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "popkv_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"POPKV_API\s+[\w\s\*]+?\b(popkv_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from popkv_b200 import _lib
    if not _lib.library_path().exists():
        from popkv_b200 import build
        build.build()
    return _lib.lib()


def test_header_declares_the_hot_path():
    names = declared_symbols()
    for name in ("popkv_pack", "popkv_query_encode", "popkv_score_encoded", "popkv_score",
                 "popkv_topk", "popkv_attn_partial", "popkv_attn_merge", "popkv_last_error",
                 "popkv_abi_version"):
        assert name in names


def test_library_exports_every_declared_symbol(lib):
    handle = ctypes.CDLL(str(ROOT / "popkv_b200" / "lib" / "libpopkv_b200.so"))
    for name in declared_symbols():
        assert hasattr(handle, name), name


def test_abi_version(lib):
    assert lib.popkv_abi_version() == 1


def _status_and_message(lib, status):
    return status, lib.popkv_last_error().decode()


def test_pack_validation_messages(lib):
    p = ctypes.c_void_p(16)
    s, msg = _status_and_message(lib, lib.popkv_pack(p, 2, 8, 10, 128, 1280, 128, p, p, p, p,
                                                     16, 0, 32, 8, None))
    assert s == 1 and "dim_group_size" in msg
    s, msg = _status_and_message(lib, lib.popkv_pack(p, 2, 8, 10, 128, 1280, 128, p, p, p, p,
                                                     16, 0, 0, 32, None))
    assert s == 1 and "token_group_size must be between 1 and 4096" in msg
    s, msg = _status_and_message(lib, lib.popkv_pack(p, 2, 8, 10, 128, 1280, 128, p, p, p, p,
                                                     12, 4, 32, 32, None))
    assert s == 2 and "capacity exceeded" in msg
    s, msg = _status_and_message(lib, lib.popkv_pack(p, 7, 8, 10, 128, 1280, 128, p, p, p, p,
                                                     16, 0, 32, 32, None))
    assert s == 1 and "fp32/fp16/bf16" in msg


def test_score_and_topk_validation_messages(lib):
    p = ctypes.c_void_p(16)
    s, msg = _status_and_message(lib, lib.popkv_score_encoded(p, p, p, p, 1, 32, p, p, p, p, 8, 100,
                                                              p, 101, 16, p, None))
    assert s == 1 and "invalid score token count" in msg
    s, msg = _status_and_message(lib, lib.popkv_score_encoded(p, p, p, p, 1, 30, p, p, p, p, 8, 100,
                                                              p, 10, 16, p, None))
    assert s == 1 and "divisible" in msg
    s, msg = _status_and_message(lib, lib.popkv_topk(p, 1, 4, 100, 100, 101, -1, p, 101, None))
    assert s == 1 and "k must be between" in msg
    s, msg = _status_and_message(lib, lib.popkv_topk(p, 0, 4, 100, 100, 10, 100, p, 10, None))
    assert s == 1 and "out_stride" in msg


def test_attention_validation_messages(lib):
    p = ctypes.c_void_p(16)
    s, msg = _status_and_message(lib, lib.popkv_attn_partial(
        p, 2, 1, 32, 128, p, p, 2, 8, 100, 0, 12800, 128, 0, 12800, 128, p, p, p, 300, None, p,
        100, p, None))
    assert s == 1 and "multiple of 16" in msg
    s, msg = _status_and_message(lib, lib.popkv_attn_partial(
        p, 2, 1, 32, 128, p, p, 2, 8, 0, 0, 12800, 128, 0, 12800, 128, p, p, p, 300, None, p,
        256, p, None))
    assert s == 1 and "non-empty prefix" in msg
    s, msg = _status_and_message(lib, lib.popkv_attn_merge(p, 4, 0, 128, p, 2, None))
    assert s == 1 and "shape mismatch" in msg


def test_peer_sum_validation_messages(lib):
    p = ctypes.c_void_p(16)
    s, msg = _status_and_message(lib, lib.popkv_peer_sum(p, 2, 3, 0, 2, p, p, p, None))  # 3 bf16: 6 bytes
    assert s == 1 and "whole 4-byte words" in msg
    s, msg = _status_and_message(lib, lib.popkv_peer_sum(p, 2, 4096, 2, 2, p, p, p, None))
    assert s == 1 and "invalid rank/world" in msg
    s, msg = _status_and_message(lib, lib.popkv_peer_sum(p, 7, 4096, 0, 2, p, p, p, None))
    assert s == 1 and "fp32/fp16/bf16" in msg
    s, msg = _status_and_message(lib, lib.popkv_peer_sum(ctypes.c_void_p(18), 2, 4096, 0, 2, p, p, p, None))
    assert s == 1 and "aligned" in msg
    s, msg = _status_and_message(lib, lib.popkv_peer_sum(None, 2, 4096, 0, 2, p, p, p, None))
    assert s == 1 and "null pointer" in msg


def test_peer_sum_rejects_partial_words_before_any_collective():
    import torch

    from popkv_b200.sharding import PeerSum
    with pytest.raises(ValueError, match="multiple of 4 bytes"):
        PeerSum(3, torch.bfloat16, "cpu")


def test_python_surface_validation_without_gpu():
    """The drop-in wrappers raise the reference's ValueErrors before touching CUDA."""
    import torch
    from popkv_b200 import popkv, popkv_cuda
    keys = torch.zeros(2, 3, 128)
    with pytest.raises(ValueError, match="contiguous CUDA"):
        popkv_cuda.pack_keys(keys)
    with pytest.raises(ValueError, match="dim_group_size must be one of 16, 32, 64"):
        popkv_cuda._validate_dim_group_size(8)
    with pytest.raises(ValueError, match="requires dim_group_size=64"):
        popkv_cuda._validate_dim_kernel(16, "g64-u64")
    with pytest.raises(ValueError):
        popkv.RetrievalConfig(budget=1).validate()
    popkv.RetrievalConfig(group_size=500).validate()
    with pytest.raises(ValueError, match="non-specialized"):
        popkv.RetrievalConfig(group_size=500, dim_group_size=16).validate()
    assert popkv.POPKV_PRESETS == {"popkv-normal": (32, 32), "popkv-q": (128, 16), "popkv-s": (64, 64)}
    out = popkv._append_current(torch.tensor([[4, 7], [2, 9]]), 12)
    assert out[:, -1].tolist() == [11, 11]
    with pytest.raises(NotImplementedError):
        popkv_cuda.update_quest_metadata(keys, keys, keys, page=0)


def test_install_as_reference_modules():
    """The reference's lazy `from popkv_cuda import ...` / `from sparse_kernels import ...` resolve here."""
    import sys
    import popkv_b200
    saved = {n: sys.modules.get(n) for n in ("popkv_cuda", "sparse_kernels")}
    try:
        for n in saved:
            sys.modules.pop(n, None)
        popkv_b200.install_as_reference_modules()
        from popkv_cuda import pack_keys, pack_keys_into, query_encode, score_encoded  # noqa: F401
        from sparse_kernels import (indexed_attention_split_merge,  # noqa: F401
                                    indexed_attention_split_partial)
        assert pack_keys is popkv_b200.popkv_cuda.pack_keys
        assert indexed_attention_split_partial is popkv_b200.sparse_kernels.indexed_attention_split_partial
        popkv_b200.install_as_reference_modules()  # idempotent
        sys.modules["popkv_cuda"] = type(sys)("popkv_cuda")
        with pytest.raises(RuntimeError, match="already imported"):
            popkv_b200.install_as_reference_modules()
    finally:
        for n, m in saved.items():
            if m is None:
                sys.modules.pop(n, None)
            else:
                sys.modules[n] = m


def test_ctypes_signatures_match_the_header():
    """Every declared entry point is bound with the header's argument count."""
    from popkv_b200 import _lib
    text = HEADER.read_text()
    for m in re.finditer(r"POPKV_API\s+[\w\s\*]+?\b(popkv_\w+)\s*\(([^;]*?)\)\s*;", text, re.S):
        name, params = m.group(1), m.group(2).strip()
        count = 0 if params in ("", "void") else params.count(",") + 1
        assert name in _lib._SIGNATURES, name
        assert len(_lib._SIGNATURES[name][0]) == count, name


def test_reference_hooks_bind():
    """The hook callables accept the reference decoder's exact calls (popkv.py:1083-1092)."""
    import inspect

    from popkv_b200 import popkv as P
    from popkv_b200 import popkv_cuda as C
    # scorer(encoded_query, packed, head_to_kv=..., tokens=..., dim_group_size=..., dim_kernel=...)
    inspect.signature(C.score_encoded).bind(
        object(), object(), head_to_kv=object(), tokens=1, dim_group_size=16, dim_kernel="g16")
    # experimental_topk(scores, k), positional
    inspect.signature(P.topk).bind(object(), 7)
    with pytest.raises(TypeError):
        inspect.signature(P.topk).bind(object())


def test_score_dispatch_switch_validation(lib):
    """popkv_score_dispatch takes 0 (auto), 1 (popcount) or 2 (fp8) and rejects anything else."""
    from popkv_b200 import popkv_cuda as C
    status, message = _status_and_message(lib, lib.popkv_score_dispatch(3))
    assert status == 1 and "mode must be" in message  # POPKV_ERR_INVALID
    with pytest.raises(ValueError):
        C.set_score_dispatch("tensor")
    for mode in ("popcount", "fp8", "auto"):
        C.set_score_dispatch(mode)
