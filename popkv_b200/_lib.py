"""ctypes binding of ``libpopkv_b200.so`` (the C ABI declared in include/popkv_b200.h).

The library is the only compute path: there is no CPU or torch fallback.  If the
shared library is missing, every op raises instead of silently doing something
else.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parent / "lib" / "libpopkv_b200.so"

DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
F32, F16, BF16 = 0, 1, 2

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64

_SIGNATURES = {
    "popkv_abi_version": ([], _I),
    "popkv_last_error": ([], ctypes.c_char_p),
    "popkv_pack": ([_P, _I, _L, _L, _L, _L, _L, _P, _P, _P, _P, _L, _L, _L, _L, _P], _I),
    "popkv_append_kv": ([_P, _P, _I, _L, _L, _P, _P, _L, _L, _L, _L, _L, _P, _P, _P, _P, _L, _L, _L, _L, _P], _I),
    "popkv_query_encode": ([_P, _I, _L, _L, _L, _P, _P, _P, _P, _P], _I),
    "popkv_score_encoded": ([_P, _P, _P, _P, _L, _L, _P, _P, _P, _P, _L, _L, _P, _L, _L, _P, _P], _I),
    "popkv_score": ([_P, _I, _L, _L, _L, _P, _P, _P, _P, _L, _L, _P, _L, _L, _P, _I, _P], _I),
    "popkv_score_dispatch": ([_I], _I),
    "popkv_score_popcount": ([_P, _I, _L, _L, _L, _P, _P, _P, _P, _L, _L, _P, _L, _L, _P, _I, _P], _I),
    "popkv_score_tc": ([_P, _I, _L, _L, _L, _P, _P, _P, _P, _L, _L, _P, _L, _L, _P, _I, _P], _I),
    "popkv_topk": ([_P, _I, _L, _L, _L, _L, _L, _P, _L, _P], _I),
    "popkv_score_hist": ([_P, _I, _L, _L, _P, _P, _P, _P, _L, _L, _P, _L, _L, _P, _P, _P], _I),
    "popkv_topk_hist": ([_P, _P, _L, _L, _L, _L, _L, _P, _L, _P], _I),
    "popkv_attn_partial": ([_P, _I, _L, _L, _L, _P, _P, _I, _L, _L, _L, _L, _L, _L, _L, _L,
                            _P, _P, _P, _L, _P, _P, _L, _P, _P], _I),
    "popkv_attn_merge": ([_P, _L, _L, _L, _P, _I, _P], _I),
    "popkv_attn_partial_merge": ([_P, _I, _L, _L, _L, _P, _P, _I, _L, _L, _L, _L, _L, _L, _L, _L,
                                  _P, _P, _P, _L, _P, _P, _L, _P, _P, _P, _I, _P], _I),
    "popkv_attn_partial_merge_static": ([_P, _I, _L, _L, _L, _P, _P, _I, _L, _L, _L, _L, _L, _L, _L, _L,
                                         _P, _P, _P, _L, _P, _P, _L, _P, _I, _P], _I),
    "popkv_stage": ([_P, _P, _L, _P], _I),
    "popkv_score_tc_timeouts": ([ctypes.POINTER(ctypes.c_uint32)], _I),
    "popkv_peer_alloc": ([_L, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p], _I),
    "popkv_peer_open": ([ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)], _I),
    "popkv_peer_close": ([_P], _I),
    "popkv_peer_clear": ([_P, _L, _P], _I),
    "popkv_peer_free": ([_P], _I),
    "popkv_attn_merge_gather": ([_P, _L, _L, _L, _I, _L, _L, _P, _P, _P, _P, _P], _I),
    "popkv_peer_sum": ([_P, _I, _L, _L, _L, _P, _P, _P, _P], _I),
    "popkv_retrieve": ([_P, _I, _L, _L, _L, _P, _P, _P, _P, _L, _L, _L, _L, _L, _P, _P, _P, _I,
                        _L, _L, _L, _L, _L, _L, _P, _P, _L, _P, _P, _P, _P], _I),
    "popkv_score_dyn": ([_P, _I, _L, _L, _P, _P, _P, _P, _L, _L, _P, _P, _L, _L, _P, _L, _P], _I),
    "popkv_topk_dyn": ([_P, _L, _P, _L, _L, _L, _P, _L, _P], _I),
    "popkv_attn_dyn": ([_P, _I, _L, _L, _P, _P, _I, _L, _L, _L, _L, _L, _L, _L, _L, _P, _P, _P,
                        _P, _L, _L, _P, _L, _P, _P, _I, _P], _I),
    "popkv_append_kv_dyn": ([_P, _P, _I, _L, _L, _P, _P, _L, _L, _L, _L, _P, _L, _P, _P, _P, _P,
                             _L, _L, _L, _P], _I),
    "popkv_rms_norm": ([_P, _P, _P, _L, _L, ctypes.c_float, _P, _P], _I),
    "popkv_rope_append": ([_P, _L, _L, _L, _L, _P, _P, _P, _L, _P, _P, _P, _P, _P, _L, _L, _L,
                           _L, _L, _L, _P], _I),
    "popkv_silu_mul": ([_P, _L, _L, _P, _P], _I),
    "popkv_gemv_timeouts": ([ctypes.POINTER(ctypes.c_uint32)], _I),
    "popkv_layer_tail": ([_L, _L, _L, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_float, _P, _P, _P, _L, _L,
                          _P, _P, _P, _P, _P, _L, _P, _P, _P, _P, _P, _L, _L, _L, _L, _L, _L, _P, _L, _P,
                          _P, _P, _P, _P, _P], _I),
    "popkv_layer_tail_timeouts": ([ctypes.POINTER(ctypes.c_uint32)], _I),
    "popkv_linear": ([_P, _L, _L, _P, _L, _P, _L, _P], _I),
    "popkv_norm_qkv_rope": ([_P, _L, _L, _L, _L, _P, _P, _P, _P, _P, ctypes.c_float, _P, _P, _P, _P, _L,
                             _P, _P, _P, _P, _P, _L, _L, _L, _L, _L, _L, _P], _I),
    "popkv_norm_gate_up_swiglu": ([_P, _L, _L, _L, _P, _P, _P, ctypes.c_float, _P, _P, _P], _I),
    "popkv_norm_lm_head_argmax": ([_P, _L, _L, _L, _P, _P, _P, ctypes.c_float, _P, _P, _P, _P, _P, _P], _I),
}

_lock = threading.Lock()
_handle = None


def library_path() -> Path:
    return _LIB_PATH


def lib():
    """Load the CUDA library once; raise if it has not been built."""
    global _handle
    if _handle is None:
        with _lock:
            if _handle is None:
                if not _LIB_PATH.exists():
                    raise RuntimeError(
                        f"popkv_b200 CUDA library not found at {_LIB_PATH}; build it with "
                        "`python -m popkv_b200.build` (nvcc, sm_100a)")
                handle = ctypes.CDLL(str(_LIB_PATH))
                for name, (args, res) in _SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.argtypes = args
                    fn.restype = res
                _handle = handle
    return _handle


def check(status: int) -> None:
    """Map a C-ABI status to an exception (RuntimeError, like TORCH_CHECK)."""
    if status != 0:
        message = lib().popkv_last_error().decode("utf-8", "replace")
        raise RuntimeError(message or f"popkv_b200 call failed with status {status}")


def ptr(tensor: torch.Tensor | None):
    return None if tensor is None else ctypes.c_void_p(tensor.data_ptr())


def dtype_code(tensor: torch.Tensor) -> int:
    try:
        return DTYPE_CODES[tensor.dtype]
    except KeyError:
        raise RuntimeError(f"unsupported dtype {tensor.dtype}: expected fp32/fp16/bf16") from None


def stream_of(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
