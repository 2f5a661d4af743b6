"""Shared helpers for tests: torch <-> oracle array conversions and input builders."""
from __future__ import annotations

import numpy as np
import torch

ORACLE_DTYPE = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}


def to_oracle(t: torch.Tensor) -> tuple[np.ndarray, str]:
    """(numpy array, oracle dtype tag) of a float tensor; 16-bit types as raw bits."""
    t = t.detach().cpu()
    if t.dtype == torch.float32:
        return t.numpy(), "f32"
    return t.contiguous().view(torch.int16).numpy().view(np.uint16), ORACLE_DTYPE[t.dtype]


def bits(t: torch.Tensor) -> np.ndarray:
    """Raw 16-bit patterns of an fp16/bf16 tensor as uint16."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bits(array: np.ndarray, dtype: torch.dtype, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(array).view(np.int16)).view(dtype).to(device)


def planes_to_numpy(packed) -> tuple[np.ndarray, ...]:
    k_sign, k_mag, k_low, k_delta = packed
    return (k_sign.cpu().numpy(), k_mag.cpu().numpy(), bits(k_low), bits(k_delta))


def random_keys(gen: torch.Generator, shape, dtype, device, outliers: bool = True) -> torch.Tensor:
    x = torch.randn(*shape, generator=gen)
    if outliers:
        factors = torch.exp(torch.randn(shape[0], 1, shape[-1], generator=gen) * 0.5)
        x = x * factors
    return x.to(dtype).to(device)
