"""popkv_attn_partial_merge_static: the split attention + merge with its scratch
in the library's fixed device array (no allocation by the call).

Collected last (file name) so it also runs after every other test in one
session, when other tests have already launched the same kernels on the
device; it must pass alone as well.
"""
from __future__ import annotations

import pytest
import torch

from popkv_b200 import _lib


def _inputs(device, *, batch, q_heads, kv_heads, tokens, selected, dtype, seed):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(batch, q_heads, 128, generator=gen).to(dtype).to(device)
    keys = torch.randn(batch, kv_heads, tokens, 128, generator=gen).to(dtype).to(device)
    values = torch.randn(batch, kv_heads, tokens, 128, generator=gen).to(dtype).to(device)
    ck = torch.randn(batch, kv_heads, 128, generator=gen).to(dtype).to(device)
    cv = torch.randn(batch, kv_heads, 128, generator=gen).to(dtype).to(device)
    idx = torch.randint(tokens, (batch, q_heads, selected), generator=gen).to(device)
    idx[..., -1] = tokens  # the current slot
    mapping = (torch.arange(q_heads) // (q_heads // kv_heads)).to(device)
    return q, keys, values, ck, cv, idx, mapping


def _args(q, keys, values, ck, cv, idx, mapping, split):
    code = _lib.dtype_code(q)
    return [_lib.ptr(q), code, q.shape[0], q.shape[1], 128, _lib.ptr(keys), _lib.ptr(values), code,
            keys.shape[1], keys.shape[2], keys.stride(0), keys.stride(1), keys.stride(2),
            values.stride(0), values.stride(1), values.stride(2), _lib.ptr(ck), _lib.ptr(cv),
            _lib.ptr(idx), idx.shape[2], None, _lib.ptr(mapping), split]


@pytest.mark.gpu
@pytest.mark.parametrize("batch,q_heads,kv_heads,tokens,selected,dtype,split", [
    (1, 32, 8, 32768, 4096, torch.bfloat16, 256),   # single launch, last CTA merges
    (2, 8, 2, 700, 300, torch.bfloat16, 256),
    (1, 8, 2, 900, 333, torch.float16, 128),         # two-launch path on the static partials
])
def test_static_scratch_matches_caller_scratch(cuda_device, batch, q_heads, kv_heads, tokens,
                                               selected, dtype, split):
    lib = _lib.lib()
    t = _inputs(cuda_device, batch=batch, q_heads=q_heads, kv_heads=kv_heads, tokens=tokens,
                selected=selected, dtype=dtype, seed=tokens + selected)
    args = _args(*t, split)
    stream = _lib.stream_of(cuda_device)
    rows = batch * q_heads
    splits = (selected + split - 1) // split
    partials = torch.empty(rows * splits * 130, dtype=torch.float32, device=cuda_device)
    counters = torch.zeros(rows, dtype=torch.int32, device=cuda_device)
    want = torch.empty(batch, q_heads, 128, dtype=dtype, device=cuda_device)
    _lib.check(lib.popkv_attn_partial_merge(*args, _lib.ptr(partials), _lib.ptr(counters),
                                            _lib.ptr(want), _lib.dtype_code(want), stream))
    torch.cuda.synchronize()
    for _ in range(2):  # two calls in a row: the static counters must come back to zero
        out = torch.full_like(want, float("nan"))
        _lib.check(lib.popkv_attn_partial_merge_static(*args, _lib.ptr(out), _lib.dtype_code(out),
                                                       stream))
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert (out.float() - want.float()).abs().max().item() <= 2 ** -7


def test_static_scratch_rejects_sizes_beyond_its_limit():
    """Oversized calls fail with POPKV_ERR_CAPACITY before any CUDA call (no GPU needed)."""
    if not _lib.library_path().exists():
        from popkv_b200 import build
        build.build()
    lib = _lib.lib()
    base = [None, _lib.BF16, 1, 65537, 128, None, None, _lib.BF16, 1, 1000, 0, 0, 128, 0, 0, 128,
            None, None, None, 100, None, None, 256, None, _lib.BF16, None]
    assert lib.popkv_attn_partial_merge_static(*base) == 2
    assert b"static scratch" in lib.popkv_last_error()
    # 32 rows x 2048 splits x 130 fp32 > 2^20.
    base[3], base[19], base[22] = 32, 2048 * 16, 16
    assert lib.popkv_attn_partial_merge_static(*base) == 2
    assert b"static scratch" in lib.popkv_last_error()
