"""Seeded synthetic decode-step inputs with the reference benchmarks' shapes.

The reference measures PopKV on Llama-3.1-8B activations from PG19/LongBench
text; neither the gated weights nor the datasets are available here, so the
benchmarks and tests use these stand-ins with the same shapes and the value
distributions the benchmark configuration names:

* keys:    N(0, 1) per element, times a per-(KV head, channel) factor
           exp(N(0, 0.5)) that creates outlier channels, then RoPE at the
           token's position (theta 500000);
* queries: N(0, 1), RoPE at position ``context`` (the decoded token);
* values:  N(0, 1);
* the current token's key/value follow the key/value rules at position
  ``context``.

Everything is drawn in float32 from ``numpy.random.Generator(PCG64(seed))`` in
a fixed order (RoPE tables in float64, rounded to float32), so every machine
(and the CPU oracle) sees identical inputs.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

ROPE_THETA = 500000.0


def rope_tables(positions: np.ndarray, head_dim: int, theta: float = ROPE_THETA):
    """cos/sin tables [len(positions), head_dim] of Llama's rotate-half RoPE."""
    inv_freq = 1.0 / theta ** (np.arange(0, head_dim, 2, dtype=np.float64) / head_dim)
    angles = np.asarray(positions, dtype=np.float64)[:, None] * inv_freq[None, :]
    emb = np.concatenate([angles, angles], axis=-1)
    return np.cos(emb), np.sin(emb)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    half = x.shape[-1] // 2
    out = x * cos
    out[..., :half] -= x[..., half:] * sin[..., :half]
    out[..., half:] += x[..., :half] * sin[..., half:]
    return out


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float values to bfloat16 (nearest-even); returns the uint16 patterns."""
    bits = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = (bits + (np.uint32(0x7FFF) + ((bits >> np.uint32(16)) & np.uint32(1)))) >> np.uint32(16)
    return rounded.astype(np.uint16)


def bf16_bits_to_float(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


@dataclass
class DecodeInputs:
    """One decode step of one attention layer (arrays are float32 values).

    keys/values: [batch, kv_heads, context, head_dim]; queries: [batch, q_heads,
    head_dim]; current_keys/current_values: [batch, kv_heads, head_dim].
    When ``dtype == "bf16"`` the float32 arrays hold bf16-representable values
    and ``bits()`` returns their 16-bit patterns.
    """
    keys: np.ndarray
    values: np.ndarray
    queries: np.ndarray
    current_keys: np.ndarray
    current_values: np.ndarray
    dtype: str

    def bits(self, name: str) -> np.ndarray:
        if self.dtype != "bf16":
            raise ValueError("bits() is only defined for bf16 workloads")
        return to_bf16_bits(getattr(self, name))


def decode_inputs(*, batch: int = 1, q_heads: int = 32, kv_heads: int = 8, head_dim: int = 128,
                  context: int = 4096, seed: int = 0, dtype: str = "bf16") -> DecodeInputs:
    if dtype not in ("f32", "bf16"):
        raise ValueError("dtype must be 'f32' or 'bf16'")
    rng = np.random.Generator(np.random.PCG64(seed))
    f32 = np.float32
    cos, sin = (t.astype(f32) for t in rope_tables(np.arange(context + 1), head_dim))
    factors = np.exp(rng.normal(0.0, 0.5, size=(batch, kv_heads, 1, head_dim))).astype(f32)
    keys = rng.standard_normal((batch, kv_heads, context, head_dim), dtype=f32)
    keys *= factors
    keys = apply_rope(keys, cos[:context], sin[:context])
    values = rng.standard_normal((batch, kv_heads, context, head_dim), dtype=f32)
    queries = apply_rope(rng.standard_normal((batch, q_heads, head_dim), dtype=f32),
                         cos[context], sin[context])
    current_keys = apply_rope(rng.standard_normal((batch, kv_heads, head_dim), dtype=f32)
                              * factors[:, :, 0], cos[context], sin[context])
    current_values = rng.standard_normal((batch, kv_heads, head_dim), dtype=f32)
    arrays = [keys, values, queries, current_keys, current_values]
    if dtype == "bf16":
        arrays = [bf16_bits_to_float(to_bf16_bits(a)) for a in arrays]
    return DecodeInputs(*arrays, dtype=dtype)


def head_to_kv(q_heads: int, kv_heads: int) -> np.ndarray:
    """GQA mapping arange(QH) // (QH / KVH) (popkv.py:783)."""
    return np.arange(q_heads, dtype=np.int64) // (q_heads // kv_heads)
