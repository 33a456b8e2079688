"""Test helpers: numpy <-> torch conversion keeping bf16 as uint16 bit patterns."""

from __future__ import annotations

import numpy as np
import torch

NP_OF = {"float32": np.float32, "float16": np.float16, "bfloat16": np.uint16}
TORCH_OF = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def to_torch(a: np.ndarray, dtype: str | None = None, device="cuda") -> torch.Tensor:
    a = np.ascontiguousarray(a)
    if dtype == "bfloat16":
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(device)
    return torch.from_numpy(a.copy()).to(device)


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype in (getattr(torch, "float8_e4m3fn", None), getattr(torch, "float8_e5m2", None)):
        return t.view(torch.uint8).numpy()
    return t.numpy()


def same_bits(a, b) -> bool:
    a = to_np(a) if isinstance(a, torch.Tensor) else np.ascontiguousarray(a)
    b = to_np(b) if isinstance(b, torch.Tensor) else np.ascontiguousarray(b)
    return a.shape == b.shape and a.dtype.itemsize == b.dtype.itemsize and a.tobytes() == b.tobytes()


def first_diff(a, b) -> str:
    a = to_np(a) if isinstance(a, torch.Tensor) else np.asarray(a)
    b = to_np(b) if isinstance(b, torch.Tensor) else np.asarray(b)
    if a.shape != b.shape:
        return f"shape {a.shape} vs {b.shape}"
    av = a.view(np.uint8 if a.dtype.itemsize == 1 else (np.uint16 if a.dtype.itemsize == 2 else np.uint32))
    bv = b.view(av.dtype)
    idx = np.argwhere(av != bv)
    if idx.size == 0:
        return "equal"
    i = tuple(idx[0])
    return f"{len(idx)} differing elements; first at {i}: {a[i]!r} vs {b[i]!r}"
