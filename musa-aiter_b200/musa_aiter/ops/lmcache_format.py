"""Describe LMCache memory tensors and SGLang split lists as layout specs.

Reference contract: musa_aiter/ops/lmcache_format.py:12-139 (format names,
shape rules and messages).
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from typing import Sequence

import torch

from .kv_layout import KVLayoutKind, KVLayoutSpec, KVOrganization


class LMCacheFormat(str, Enum):
    KV_2LTD = "kv_2ltd"
    KV_T2D = "kv_t2d"
    KV_2TD = "kv_2td"
    SGLANG_SPLIT_LIST = "sglang_split_list"


@dataclass(frozen=True)
class LMCacheFormatFacts:
    format: LMCacheFormat
    spec: KVLayoutSpec


_DTYPES = (torch.float32, torch.float16, torch.bfloat16, torch.uint8)


def _check_dtype(t: torch.Tensor) -> None:
    if t.dtype not in _DTYPES:
        raise ValueError(f"unsupported LMCache dtype={t.dtype}")


def _dtype_name(t: torch.Tensor) -> str:
    return str(t.dtype).removeprefix("torch.")


def _linear(t: torch.Tensor, kind: KVLayoutKind, org: KVOrganization, layers: int, tokens: int, hidden: int) -> KVLayoutSpec:
    return KVLayoutSpec.linear(num_layers=layers, num_tokens=tokens, num_heads=1, head_size=hidden,
                               dtype_name=_dtype_name(t), organization=org, kind=kind, device_kind=t.device.type)


def describe_lmcache_format(memory_tensor: torch.Tensor) -> LMCacheFormatFacts:
    """``[2, NL, T, H]`` -> KV_2LTD; ``[T, 2, H]`` -> KV_T2D; ``[2, T, H]`` -> KV_2TD."""
    if not isinstance(memory_tensor, torch.Tensor) or not memory_tensor.is_contiguous():
        raise ValueError("LMCache memory tensor must be contiguous")
    t = memory_tensor
    if t.dim() == 4:
        if t.shape[0] != 2:
            raise ValueError("KV_2LTD memory tensor must have leading K/V dimension 2")
        _check_dtype(t)
        _, layers, tokens, hidden = map(int, t.shape)
        return LMCacheFormatFacts(LMCacheFormat.KV_2LTD, _linear(t, KVLayoutKind.KV_2LTD, KVOrganization.SEPARATE, layers, tokens, hidden))
    if t.dim() != 3:
        raise ValueError("LMCache memory tensor rank must be 3 or 4")
    first, second, hidden = int(t.shape[0]), int(t.shape[1]), int(t.shape[-1])
    _check_dtype(t)
    if first == 2 and second == 2:
        raise ValueError("3-D LMCache tensor is ambiguous when both leading dimensions are 2")
    if second == 2:
        return LMCacheFormatFacts(LMCacheFormat.KV_T2D, _linear(t, KVLayoutKind.KV_T2D, KVOrganization.MERGED, 1, first, hidden))
    if first == 2:
        return LMCacheFormatFacts(LMCacheFormat.KV_2TD, _linear(t, KVLayoutKind.KV_2TD, KVOrganization.SEPARATE, 1, second, hidden))
    raise ValueError("3-D LMCache memory tensor must be [T, 2, H] or [2, T, H]")


def describe_sglang_split_list(kvcaches: Sequence[Sequence[torch.Tensor]]) -> LMCacheFormatFacts:
    """``[K_layers, V_layers]`` of ``[NB, BS, NH, HS]`` tensors -> TWO_X_NL spec (2*NL pointers)."""
    if len(kvcaches) != 2:
        raise ValueError("SGLang split-list must contain K and V layer lists")
    if not kvcaches[0] or not kvcaches[1]:
        raise ValueError("SGLang split-list must be non-empty")
    if len(kvcaches[0]) != len(kvcaches[1]):
        raise ValueError("SGLang K/V layer lists must have the same length")
    first = kvcaches[0][0]
    if not isinstance(first, torch.Tensor) or first.dim() != 4:
        raise ValueError("SGLang split-list entries must be [NB, BS, NH, HS] tensors")
    _check_dtype(first)
    nb, bs, nh, hs = map(int, first.shape)
    for axis in kvcaches:
        for t in axis:
            if not isinstance(t, torch.Tensor) or t.shape != first.shape:
                raise ValueError("all SGLang split-list entries must share one shape")
            if t.dtype != first.dtype:
                raise ValueError("all SGLang split-list entries must share one dtype")
    row = nh * hs * first.element_size()
    spec = KVLayoutSpec(kind=KVLayoutKind.TWO_X_NL, num_layers=len(kvcaches[0]), num_blocks=nb, block_size=bs, num_heads=nh,
                        head_size=hs, row_bytes=row, block_stride_bytes=bs * row, dtype_name=_dtype_name(first),
                        organization=KVOrganization.SPLIT_LIST, is_contiguous=False,
                        pointer_table_length=2 * len(kvcaches[0]), device_kind=first.device.type)
    return LMCacheFormatFacts(LMCacheFormat.SGLANG_SPLIT_LIST, spec)
